"""The allocation-free attention entry point, checked against the ordinary one.

``mes_varlen_attention_noalloc`` exists for callers that cannot allocate device memory
(an FFI caller holding only the buffers its runtime gave it, or a serving process whose
device memory is fixed by its own pool); it keeps the schedule workspace in a fixed array
inside the library.  This file is collected last on purpose, and each test calls the
entry point twice in a row on different batches, because the array keeps the previous
call's contents.

Both entry points run the same schedule and attention kernels on the same work list, so
their outputs must be identical bit for bit; the output buffer is filled with NaN before
each call, so a row the kernel never wrote fails the comparison.  The result is also
checked against the CPU oracle (per-sequence causal SDPA in fp32) at the attention tests'
tolerance of 1e-2 relative to max|O|.
"""
import ctypes

import pytest
import torch

from mes_b200 import _C, synthetic
from oracle import ops as oops

pytestmark = pytest.mark.gpu
DEV = "cuda"
D = 128


def _noalloc(positions, qkv, Hq, Hkv):
    T = positions.shape[0]
    out = torch.full((T, Hq * D), float("nan"), dtype=torch.bfloat16, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = _C.lib().mes_varlen_attention_noalloc(
        ctypes.c_void_p(positions.data_ptr()), ctypes.c_void_p(qkv.data_ptr()), qkv.stride(0),
        ctypes.c_void_p(out.data_ptr()), T, Hq, Hkv, D, D ** -0.5, stream)
    assert st == 0, _C.status_string(st)
    return out


def _case(lengths, Hq, Hkv, seed):
    _, pos, _ = synthetic.packed_batch(lengths, 100)
    positions = torch.from_numpy(pos).to(DEV)
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(len(pos), (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16).to(DEV)
    return positions, qkv


def test_noalloc_matches_workspace_entry_point_twice():
    for lengths, Hq, Hkv, seed in [([300, 1000, 5, 129], 16, 8, 1), ([64, 7, 513], 12, 2, 2)]:
        positions, qkv = _case(lengths, Hq, Hkv, seed)
        T = positions.shape[0]
        want = torch.full((T, Hq * D), float("nan"), dtype=torch.bfloat16, device=DEV)
        _C.varlen_attention(qkv, _C.varlen_schedule(positions), Hq, Hkv, D, D ** -0.5, out=want)
        got = _noalloc(positions, qkv, Hq, Hkv)
        torch.cuda.synchronize()
        assert not torch.isnan(want).any()
        assert torch.equal(got, want), lengths
        q, k, v = qkv.float().cpu().split([Hq * D, Hkv * D, Hkv * D], dim=1)
        ref = oops.varlen_causal_attention(q, k, v, oops.cu_seqlens_from_positions(positions.cpu()),
                                           Hq, Hkv, D)
        err = (got.float().cpu() - ref).abs().max().item()
        assert err <= 1e-2 * ref.abs().max().item(), err
    assert _C.take_device_error() == 0


def test_noalloc_rejects_batches_over_its_limit():
    limit = _C.lib().mes_varlen_attention_noalloc_max_tokens()
    assert limit == 131072
    positions, qkv = _case([16], 2, 1, 3)
    st = _C.lib().mes_varlen_attention_noalloc(
        ctypes.c_void_p(positions.data_ptr()), ctypes.c_void_p(qkv.data_ptr()), qkv.stride(0),
        ctypes.c_void_p(qkv.data_ptr()), limit + 1, 2, 1, D, 1.0, None)
    assert st == 1  # MES_ERR_INVALID, before anything is launched
