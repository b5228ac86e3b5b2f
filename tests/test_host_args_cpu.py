"""The torch-facing wrappers' host checks, on CPU.  The library's launch entry points are
replaced by a recorder (its size queries stay the real library's): every call the model
makes in a forward passes the checks, and a tensor on another device, of another dtype or
of another shape is refused before any pointer reaches the library.  At tensor parallelism 2
(two ``gloo`` ranks) the overlapped forward's calls pass them too."""
import datetime
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import __graft_entry__  # noqa: E402  (spawned ranks import this module by name)

__graft_entry__.load_package()

from mes_b200 import _C, synthetic  # noqa: E402
from mes_b200.models import Qwen2ForCausalLM, Qwen3ForCausalLM  # noqa: E402
from mes_b200.schemas.config import MESConfig  # noqa: E402

_REAL = ("mes_varlen_workspace_size", "mes_awq_gemm_workspace_size", "mes_status_string")


class _RecordingLib:
    def __init__(self, real):
        self.real = real
        self.calls = []
        self.reserve = []        # values given to mes_set_sm_reserve

    def __getattr__(self, name):
        if name in _REAL:
            return getattr(self.real, name)

        def launch(*args):
            self.calls.append(name)
            if name == "mes_set_sm_reserve":
                self.reserve.append(args[0])
            return 0
        return launch


@pytest.fixture
def rec(monkeypatch):
    fake = _RecordingLib(_C.lib())
    monkeypatch.setattr(_C, "lib", lambda: fake)
    monkeypatch.setattr(_C, "_stream", lambda t: 0)
    return fake


@pytest.mark.parametrize("cls,cfg", [
    (Qwen3ForCausalLM, synthetic.qwen3_0_6b(num_hidden_layers=2, vocab_size=1000)),
    (Qwen2ForCausalLM, synthetic.qwen2_1_5b(num_hidden_layers=2, vocab_size=1000)),
])
@pytest.mark.parametrize("lengths", [[300, 200, 1], [1000, 700, 500]])   # fused / panel GEMMs
def test_model_forward_calls_pass_the_checks(rec, cls, cfg, lengths):
    model = cls(MESConfig(model_config=cfg))
    ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size)
    ids, pos, last = map(torch.from_numpy, (ids, pos, last))
    out = model(ids, pos)
    assert out.shape == (len(ids), cfg.hidden_size) and out.dtype == torch.bfloat16
    rows = model.forward_last_rows(ids, pos, last)
    assert rows.shape == (len(lengths), cfg.hidden_size)
    emb = _C.last_token_l2(out, last)
    assert emb.shape == (len(lengths), cfg.hidden_size) and emb.dtype == torch.float32
    # (tp = 1: o_proj and down_proj add into the fp32 residual in their GEMM epilogue, so
    # every norm reads the residual alone)
    want = {"mes_varlen_schedule", "mes_embedding_f32", "mes_rmsnorm_f32in", "mes_qknorm_rope",
            "mes_varlen_attention", "mes_awq_repack", "mes_awq_gemm_ws", "mes_last_token_l2"}
    if sum(lengths) > 1024:
        want |= {"mes_awq_panels", "mes_awq_gemm_on_panel"}
    assert want <= set(rec.calls), want - set(rec.calls)


def _awq(K=256, N=128):
    return (torch.zeros(K // 8, N, dtype=torch.int32), torch.zeros(K // 128, N // 8, dtype=torch.int32),
            torch.zeros(K // 128, N, dtype=torch.int16))


def test_bad_arguments_are_refused_before_the_library(rec):
    T, H, D = 16, 256, 128
    x = torch.zeros(T, H, dtype=torch.bfloat16)
    w = torch.ones(H, dtype=torch.bfloat16)
    qw, qz, sc = _awq()
    xa = torch.zeros(T, 256, dtype=torch.bfloat16)
    pos = torch.arange(T)
    qkv = torch.zeros(T, 4 * D, dtype=torch.bfloat16)
    cache = torch.zeros(64, D)
    ws = _C.varlen_schedule(pos)
    bad = [
        lambda: _C.rmsnorm(x, w.to("meta"), 1e-6),                     # another device
        lambda: _C.rmsnorm(x, w.float(), 1e-6),                         # fp32 weight
        lambda: _C.rmsnorm(x, w[:128], 1e-6),                           # short weight
        lambda: _C.rmsnorm(x, w, 1e-6, torch.empty(T, H)),              # fp32 out
        lambda: _C.add_rmsnorm_f32res(x, torch.zeros(T, H, device="meta"), w, 1e-6),
        lambda: _C.add_rmsnorm(x, x.clone(), w, 1e-6, residual_out=torch.empty(T, H - 8, dtype=torch.bfloat16)),
        lambda: _C.embedding(torch.zeros(T, dtype=torch.int64), x, torch.empty(T, H)),
        lambda: _C.embedding_f32(torch.zeros(T, dtype=torch.int64, device="meta"), x),
        lambda: _C.silu_mul(x, torch.empty(T, H, dtype=torch.bfloat16)),
        lambda: _C.qknorm_rope(qkv[:8], pos, cache, 2, 1, D),           # rows != positions
        lambda: _C.qknorm_rope(qkv, pos, cache[:, :64], 2, 1, D),       # cache width != D
        lambda: _C.qknorm_rope(qkv, pos, cache, 2, 1, D, torch.ones(D), torch.ones(D)),
        lambda: _C.varlen_attention(qkv, ws[:64], 2, 1, D, 0.1),         # workspace too small
        lambda: _C.varlen_attention(qkv, ws, 2, 1, D, 0.1, torch.empty(T, 2 * D)),
        lambda: _C.last_token_l2(x, torch.zeros(2, 1, dtype=torch.int64)),
        lambda: _C.last_token_l2(x, torch.zeros(2, dtype=torch.int64), torch.empty(2, H - 1)),
        lambda: _C.awq_gemm(xa, qw, qz, sc.float()),                    # fp32 scales
        lambda: _C.awq_gemm(xa, qw, qz[:, :8], sc),                     # qzeros of another N
        lambda: _C.awq_gemm(xa, qw, qz, sc[:1]),                        # scales of another K
        lambda: _C.awq_gemm(xa, qw, qz, sc, torch.zeros(64, dtype=torch.bfloat16)),   # short bias
        lambda: _C.awq_gemm(xa, qw, qz, sc, None, torch.empty(T, 128)),  # fp32 out
        lambda: _C.awq_gemm(xa, qw.t().contiguous().t(), qz, sc),        # strided qweight
        lambda: _C.awq_gemm_silu(xa, qw, qz, sc, torch.empty(T, 128, dtype=torch.bfloat16)),
        lambda: _C.awq_gemm_residual(xa, qw, qz, sc, torch.zeros(T, 128, device="meta")),
        lambda: _C.awq_dequant(qw, qz.to(torch.int16), sc),
        lambda: _C.awq_panels([(qw, qz, sc)], [torch.empty(128, 128, dtype=torch.bfloat16)]),
    ]
    rec.calls.clear()
    for i, call in enumerate(bad):
        with pytest.raises(_C.MesError):
            call()
        assert rec.calls == [], (i, rec.calls)
    # The same calls with valid arguments reach the library.
    _C.rmsnorm(x, w, 1e-6)
    _C.qknorm_rope(qkv, pos, cache, 2, 1, D, torch.ones(D, dtype=torch.bfloat16),
                   torch.ones(D, dtype=torch.bfloat16))
    _C.varlen_attention(qkv, ws, 2, 1, D, 0.1)
    _C.awq_gemm(xa, qw, qz, sc, torch.zeros(128, dtype=torch.bfloat16))
    _C.awq_panels([(qw, qz, sc)], [torch.empty(128, 256, dtype=torch.bfloat16)])
    assert rec.calls == ["mes_rmsnorm", "mes_qknorm_rope", "mes_varlen_attention",
                         "mes_awq_gemm_ws", "mes_awq_panels"]


def _tp_rank(rank, world, port, q):
    import torch.distributed as dist
    from mes_b200.models import qwen2
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        fake = _RecordingLib(_C.lib())
        _C.lib = lambda: fake
        _C._stream = lambda t: 0
        cfg = synthetic.qwen3_0_6b(num_hidden_layers=2, vocab_size=1000)
        model = Qwen3ForCausalLM(MESConfig(model_config=cfg))
        ids, pos, _ = synthetic.packed_batch([1000] * 5, cfg.vocab_size)
        split = qwen2.DecoderModel.overlap_split_host(pos)
        out = model(torch.from_numpy(ids), torch.from_numpy(pos), split)
        q.put((rank, split, tuple(out.shape), fake.reserve, sorted(set(fake.calls))))
    finally:
        dist.destroy_process_group()


def test_tp2_overlapped_forward_calls_pass_the_checks():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [q.get(timeout=10) for _ in procs]
    for rank, split, shape, reserve, calls in results:
        assert split == 2000 and shape == (5000, 1024), (rank, split, shape)
        # The persistent kernels leave 16 SMs to NCCL during the overlap, then all of them.
        assert reserve == [16, 0], reserve
        # Micro-batches of 2000 / 3000 tokens: panel GEMMs; the bf16 partial products are
        # all-reduced, then added into the residual by the add + RMSNorm kernel.
        assert {"mes_awq_panels", "mes_awq_gemm_on_panel", "mes_add_rmsnorm_f32res",
                "mes_varlen_attention", "mes_qknorm_rope"} <= set(calls), calls
