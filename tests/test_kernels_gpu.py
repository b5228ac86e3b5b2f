"""Parity of each CUDA kernel (called through the C ABI) against the CPU oracle."""
import numpy as np
import pytest
import torch

from mes_b200 import _C, synthetic
from oracle import awq as oawq
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16(x):
    return x.to(torch.bfloat16)


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> int:
    """Largest distance between two bf16 tensors in units in the last place."""
    def key(t):
        i = t.to(torch.bfloat16).view(torch.int16).to(torch.int64)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return int((key(a) - key(b)).abs().max())


def ulp_close(a: torch.Tensor, b: torch.Tensor, ulps: int = 1) -> bool:
    d = ulp_diff(a, b)
    assert d <= ulps, f"{d} ulps apart (allowed {ulps})"
    return True


def test_no_device_error_at_start():
    assert _C.take_device_error() == 0


def test_bounded_wait_runs_out_and_reports_timeout():
    # The library's bounded mbarrier wait, made to run out on purpose: a 1 ms limit on a
    # phase nothing completes.  The kernel records MES_ERR_TIMEOUT and returns; the
    # context stays usable.  With the arrival made first, nothing is recorded.
    stream = torch.cuda.current_stream().cuda_stream
    assert _C.lib().mes_wait_probe(1_000_000, 1, stream) == 0
    assert _C.take_device_error() == 0
    assert _C.lib().mes_wait_probe(1_000_000, 0, stream) == 0
    assert _C.take_device_error() == 4          # MES_ERR_TIMEOUT
    assert _C.take_device_error() == 0          # taking the error cleared it
    x = torch.randn(8, 32, device=DEV).to(torch.bfloat16)
    assert ulp_close(_C.silu_mul(x).cpu(), bf16(ops.silu_and_mul(x.cpu().float())), 1)


# ------------------------------------------------------------------------------ AWQ
@pytest.mark.parametrize("K,N,seed", [(128, 128, 0), (256, 384, 1), (1024, 1024, 2)])
def test_awq_repack_and_dequant_bit_exact(K, N, seed):
    qw, qz, sc = oawq.random_awq(K, N, seed=seed)
    qw_mes = _C.awq_repack(torch.from_numpy(qw).to(DEV))
    assert np.array_equal(qw_mes.cpu().numpy(), oawq.mes_repack(qw))
    w = _C.awq_dequant(qw_mes, torch.from_numpy(qz).to(DEV),
                       torch.from_numpy(sc).view(torch.int16).to(DEV))
    want = oawq.dequant_bf16_bits(qw, qz, sc)          # [K, N] bf16 bits
    got = w.cpu().view(torch.int16).numpy().view(np.uint16).T  # W^T [N, K] -> [K, N]
    assert np.array_equal(got, want)


def test_awq_dequant_exhaustive_codes_and_edge_scales():
    # every (q, z) pair against scales covering rounding ties, subnormal fp16, tiny/huge
    K, N = 256, 256
    q = np.tile(np.arange(16, dtype=np.uint8), (K, N // 16))
    rng = np.random.default_rng(7)
    q = rng.permuted(q, axis=1)
    z = np.repeat(np.arange(16, dtype=np.uint8)[None, :], K // 128 * N // 16, 0).reshape(K // 128, N)
    edge = np.array([1e-7, 6e-8, 6.1e-5, 0.002, 0.00201, 0.0199, 0.02, 0.5, 1.0, 1.0009766,
                     3.14159, 65504.0, 0.33333, 0.1, 7e-3, 2.0 ** -14], dtype=np.float16)
    s = rng.choice(edge, size=(K // 128, N)).astype(np.float16)
    qw, qz = oawq.awq_pack(q), oawq.awq_pack(z)
    qw_mes = _C.awq_repack(torch.from_numpy(qw).to(DEV))
    w = _C.awq_dequant(qw_mes, torch.from_numpy(qz).to(DEV), torch.from_numpy(s).view(torch.int16).to(DEV))
    got = w.cpu().view(torch.int16).numpy().view(np.uint16).T
    assert np.array_equal(got, oawq.dequant_bf16_bits(qw, qz, s))


def _gemm_case(M, K, N, bias, seed):
    qw, qz, sc = oawq.random_awq(K, N, seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16) if bias else None
    w = torch.from_numpy(oawq.bf16_bits_to_f32(oawq.dequant_bf16_bits(qw, qz, sc)))  # [K, N]
    ref = x.float() @ w
    if b is not None:
        ref = ref + b.float()
    qw_mes = _C.awq_repack(torch.from_numpy(qw).to(DEV))
    y = _C.awq_gemm(x.to(DEV), qw_mes, torch.from_numpy(qz).to(DEV),
                    torch.from_numpy(sc).view(torch.int16).to(DEV),
                    None if b is None else b.to(DEV))
    return y.float().cpu(), ref


@pytest.mark.parametrize("M,K,N,bias", [
    (1, 128, 128, False), (16, 256, 256, True), (17, 1024, 128, False), (64, 512, 384, True),
    (100, 1024, 256, False), (128, 256, 128, False), (129, 1024, 512, True),
    (300, 2048, 1024, False), (1000, 1024, 6144, False), (777, 3072, 1024, True),
    (200, 1024, 19456, True)])
def test_awq_gemm_matches_fp32(M, K, N, bias):
    # Tolerance: fp32 accumulation order and one bf16 rounding of the output.
    y, ref = _gemm_case(M, K, N, bias, seed=M + K + N)
    err = (y - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-2 * scale + 1e-3, (err, scale)
    cos = torch.nn.functional.cosine_similarity(y, ref, dim=1)
    assert cos.min().item() > 0.9999


def test_awq_gemm_rejects_bad_shapes():
    x = torch.zeros(4, 100, dtype=torch.bfloat16, device=DEV)
    qw = torch.zeros(100 // 8, 128, dtype=torch.int32, device=DEV)
    with pytest.raises(_C.MesError):
        _C.awq_gemm(x, qw, torch.zeros(1, 16, dtype=torch.int32, device=DEV),
                    torch.zeros(1, 128, dtype=torch.int16, device=DEV))


# ------------------------------------------------------------------------------ norms
@pytest.mark.parametrize("rows,H", [(1, 1024), (37, 1024), (513, 1536), (64, 4096)])
def test_rmsnorm_and_add_rmsnorm(rows, H):
    g = torch.Generator().manual_seed(rows + H)
    x = bf16(torch.randn(rows, H, generator=g))
    r = bf16(torch.randn(rows, H, generator=g))
    w = bf16(1 + 0.1 * torch.randn(H, generator=g))
    # Tolerance: the kernel's fp32 rsqrt may move the first of the two bf16 roundings
    # (normalised value, then * weight) by one step -> at most 2 ulps.
    want = ops.rms_norm(x, w, 1e-6)
    got = _C.rmsnorm(x.to(DEV), w.to(DEV), 1e-6).cpu()
    assert ulp_close(got, want, 2)
    wy, wr = ops.add_rms_norm(x, r, w, 1e-6)
    xd, rd = x.to(DEV), r.to(DEV)
    gy, gr = _C.add_rmsnorm(xd, rd, w.to(DEV), 1e-6)
    assert torch.equal(gr.cpu(), wr)            # residual: one rounding of an exact fp32 sum
    assert ulp_close(gy.cpu(), wy, 2)
    # in place (the model's use): y -> x, residual_out -> residual
    _C.add_rmsnorm(xd, rd, w.to(DEV), 1e-6, out=xd, residual_out=rd)
    assert torch.equal(rd.cpu(), wr) and ulp_close(xd.cpu(), wy, 2)


# ------------------------------------------------------------------------------ rope
@pytest.mark.parametrize("norm,f32cache", [(True, False), (False, False), (True, True)])
@pytest.mark.parametrize("T,Hq,Hkv", [(300, 16, 8), (77, 12, 2), (5, 2, 1)])
def test_qknorm_rope(norm, f32cache, T, Hq, Hkv):
    D = 128
    g = torch.Generator().manual_seed(3)
    qkv = bf16(torch.randn(T, (Hq + 2 * Hkv) * D, generator=g))
    positions = torch.cat([torch.arange(100), torch.arange(150), torch.arange(50) + 4000])[:T]
    cache = ops.rope_cos_sin_cache(D, 8192, 1e6)
    cache = cache if f32cache else bf16(cache)
    qw = bf16(1 + 0.1 * torch.randn(D, generator=g))
    kw = bf16(1 + 0.1 * torch.randn(D, generator=g))
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=1)
    if norm:
        q = ops.rms_norm(q.reshape(T, Hq, D), qw, 1e-6).reshape(T, -1)
        k = ops.rms_norm(k.reshape(T, Hkv, D), kw, 1e-6).reshape(T, -1)
    want_q = ops.apply_rope(q, positions, cache, D)
    want_k = ops.apply_rope(k, positions, cache, D)
    d = qkv.to(DEV)
    _C.qknorm_rope(d, positions.to(DEV), cache.to(DEV), Hq, Hkv, D,
                   qw.to(DEV) if norm else None, kw.to(DEV) if norm else None)
    got = d.cpu()
    if norm:
        # The normalised head may differ by 2 ulps (see test_rmsnorm_and_add_rmsnorm); the
        # rotation mixes two such values, so compare with an absolute bound of 2-4 ulps of
        # the largest input magnitude.
        tol = 4 * 2.0 ** -8 * float(max(want_q.abs().max(), want_k.abs().max()))
        assert (got[:, :Hq * D].float() - want_q.float()).abs().max() <= tol
        assert (got[:, Hq * D:(Hq + Hkv) * D].float() - want_k.float()).abs().max() <= tol
    else:
        assert ulp_close(got[:, :Hq * D], want_q, 1)
        assert ulp_close(got[:, Hq * D:(Hq + Hkv) * D], want_k, 1)
    assert torch.equal(got[:, (Hq + Hkv) * D:], v)


# ------------------------------------------------------------------------------ misc
def test_silu_mul():
    g = torch.Generator().manual_seed(5)
    x = bf16(torch.randn(333, 2 * 3072, generator=g) * 3)
    want = bf16(ops.silu_and_mul(x.float()))
    got = _C.silu_mul(x.to(DEV)).cpu()
    assert ulp_close(got, want, 1)


def test_embedding_exact():
    g = torch.Generator().manual_seed(6)
    table = bf16(torch.randn(1000, 1024, generator=g))
    ids = torch.randint(0, 1000, (777,), generator=g)
    got = _C.embedding(ids.to(DEV), table.to(DEV)).cpu()
    assert torch.equal(got, ops.embedding(ids, table))
    assert _C.take_device_error() == 0


def test_last_token_l2():
    g = torch.Generator().manual_seed(8)
    hidden = bf16(torch.randn(500, 1024, generator=g))
    idx = torch.tensor([0, 99, 100, 499])
    got = _C.last_token_l2(hidden.to(DEV), idx.to(DEV)).cpu()
    want = ops.last_token_l2(hidden, idx)
    assert torch.allclose(got, want, atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("lengths", [[1], [5, 1, 1, 7], [128, 129, 127, 1000, 3],
                                     [4096, 64, 1]])
def test_varlen_schedule_cu_seqlens(lengths):
    _, pos, _ = synthetic.packed_batch(lengths, 100)
    positions = torch.from_numpy(pos)
    ws = _C.varlen_schedule(positions.to(DEV))
    cu, n = _C.varlen_cu_seqlens(ws, len(pos))
    n = int(n.item())
    want = ops.cu_seqlens_from_positions(positions)
    assert n == len(want) - 1
    assert torch.equal(cu[: n + 1].cpu().to(torch.int64), want)


# ------------------------------------------------------------------------------ attention
@pytest.mark.parametrize("lengths,Hq,Hkv", [
    ([1], 2, 1), ([5, 1, 127, 128, 129], 16, 8), ([300, 1000], 12, 2), ([257, 64, 700], 4, 4),
    ([4096, 300, 1], 32, 8), ([64, 4096], 16, 8)])
def test_varlen_attention(lengths, Hq, Hkv):
    # Tolerance 1e-2 * max|O|: P is rounded to bf16 before the PV product and O once to bf16
    # at the end; an fp32 emulation of exactly those roundings lands at 1.2e-3 (1000-token
    # sequences) and 2.1e-3 (4096) of max|O| against the fp32 reference.
    D = 128
    _, pos, _ = synthetic.packed_batch(lengths, 100)
    positions = torch.from_numpy(pos)
    T = len(pos)
    g = torch.Generator().manual_seed(T + Hq)
    qkv = bf16(torch.randn(T, (Hq + 2 * Hkv) * D, generator=g))
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=1)
    cu = ops.cu_seqlens_from_positions(positions)
    want = ops.varlen_causal_attention(q.float(), k.float(), v.float(), cu, Hq, Hkv, D)
    ws = _C.varlen_schedule(positions.to(DEV))
    got = _C.varlen_attention(qkv.to(DEV), ws, Hq, Hkv, D, D ** -0.5).float().cpu()
    assert _C.take_device_error() == 0
    err = (got - want).abs().max().item()
    assert err <= 1e-2 * want.abs().max().item(), (err, want.abs().max().item())


# ------------------------------------------------------------------ fp32 residual stream
def test_embedding_f32_exact():
    g = torch.Generator().manual_seed(16)
    table = bf16(torch.randn(500, 1536, generator=g))
    ids = torch.randint(0, 500, (333,), generator=g)
    got = _C.embedding_f32(ids.to(DEV), table.to(DEV)).cpu()
    assert got.dtype == torch.float32 and torch.equal(got, table[ids].float())


def test_embedding_many_rows_grid_stride():
    # More rows than one wave of warps holds (one warp per row, 8 rows per block, at most
    # 32 blocks per SM launched), with a 16-vector row so most lanes are idle.
    g = torch.Generator().manual_seed(18)
    table = bf16(torch.randn(100, 128, generator=g))
    ids = torch.randint(0, 100, (60000,), generator=g)
    got = _C.embedding_f32(ids.to(DEV), table.to(DEV)).cpu()
    assert torch.equal(got, table[ids].float())
    assert torch.equal(_C.embedding(ids.to(DEV), table.to(DEV)).cpu(), table[ids])
    assert _C.take_device_error() == 0


def test_rmsnorm_f32_and_add_rmsnorm_f32res():
    g = torch.Generator().manual_seed(17)
    rows, H = 257, 1024
    res = torch.randn(rows, H, generator=g) * 3
    x = bf16(torch.randn(rows, H, generator=g))
    w = bf16(1 + 0.1 * torch.randn(H, generator=g))
    # Tolerance: 2 ulps, as for the bf16 variants (fp32 rsqrt moves the first rounding).
    got = _C.rmsnorm(res.to(DEV), w.to(DEV), 1e-6).cpu()
    assert ulp_close(got, ops.rms_norm(res, w, 1e-6).to(torch.bfloat16), 2)
    rd = res.to(DEV)
    y = _C.add_rmsnorm_f32res(x.to(DEV), rd, w.to(DEV), 1e-6).cpu()
    s = x.float() + res
    assert torch.equal(rd.cpu(), s)             # fp32 residual updated exactly
    assert ulp_close(y, ops.rms_norm(s, w, 1e-6).to(torch.bfloat16), 2)


@pytest.mark.parametrize("M,K,N,bias", [(5, 256, 128, False), (130, 1024, 1024, True),
                                        (1000, 3072, 1024, False)])
def test_awq_gemm_residual_epilogue(M, K, N, bias):
    # R += X @ W (+ bias) in fp32: the bf16 rounding of the GEMM output is gone, so the
    # tolerance is that of the fp32 accumulation order alone.
    qw, qz, sc = oawq.random_awq(K, N, seed=M)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16) if bias else None
    r0 = torch.randn(M, N, generator=g)
    w = torch.from_numpy(oawq.bf16_bits_to_f32(oawq.dequant_bf16_bits(qw, qz, sc)))
    ref = r0 + x.float() @ w + (b.float() if b is not None else 0)
    rd = r0.to(DEV)
    _C.awq_gemm_residual(x.to(DEV), _C.awq_repack(torch.from_numpy(qw).to(DEV)),
                         torch.from_numpy(qz).to(DEV), torch.from_numpy(sc).view(torch.int16).to(DEV),
                         rd, None if b is None else b.to(DEV))
    err = (rd.cpu() - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item() + 1e-4, err


# ------------------------------------------------------------------ GEMM tile variants
_VARIANT_CHECK = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import __graft_entry__; __graft_entry__.load_package()
from mes_b200 import _C
from oracle import awq as oawq
# (20000, 256, 1024) spans several waves of the persistent kernels' CTAs; (600, 12288, 2048)
# has more 256-feature tiles (8) than one band of the weight panel holds (6 at K = 12288).
for M, K, N, res in [(16, 256, 256, False), (65, 256, 128, False), (300, 1024, 384, True), (777, 3072, 1024, False), (1000, 1024, 256, True), (20000, 256, 1024, True), (600, 12288, 2048, False)]:
    qw, qz, sc = oawq.random_awq(K, N, seed=M)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = torch.from_numpy(oawq.bf16_bits_to_f32(oawq.dequant_bf16_bits(qw, qz, sc)))
    ref = x.float() @ w
    args = (x.cuda(), _C.awq_repack(torch.from_numpy(qw).cuda()), torch.from_numpy(qz).cuda(),
            torch.from_numpy(sc).view(torch.int16).cuda())
    if res:
        r = torch.zeros(M, N, device="cuda")
        got = _C.awq_gemm_residual(*args, r).cpu()
        tol = 1e-4 * ref.abs().max().item() + 1e-4
    else:
        got = _C.awq_gemm(*args).float().cpu()
        tol = 1e-2 * ref.abs().max().item() + 1e-3
    err = (got - ref).abs().max().item()
    assert err <= tol, (M, K, N, res, err, tol)
for M, K, N in [(16, 256, 256), (100, 512, 384 * 2), (1000, 1024, 768)]:
    qw, qz, sc = oawq.random_awq(K, N, seed=M + 1)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = torch.from_numpy(oawq.bf16_bits_to_f32(oawq.dequant_bf16_bits(qw, qz, sc)))
    gu = x.float() @ w
    ref = torch.nn.functional.silu(gu[:, : N // 2]) * gu[:, N // 2:]
    qwi, qzi, sci = _C.interleave_gate_up(torch.from_numpy(qw).cuda(), torch.from_numpy(qz).cuda(),
                                          torch.from_numpy(sc).view(torch.int16).cuda())
    got = _C.awq_gemm_silu(x.cuda(), _C.awq_repack(qwi), qzi, sci).float().cpu()
    err = (got - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, ("silu", M, K, N, err)
assert _C.take_device_error() == 0
print("ok")
"""


@pytest.mark.parametrize("config", ["0", "1", "2", "3", "4", "panel"])
def test_awq_gemm_tile_variants(config):
    # The large-M tile variant is chosen once per process (MES_GEMM_CONFIG, MES_GEMM_PANEL),
    # so each runs in a child process: the fused dequantising kernels (0-4, weight panel
    # off) and the dequantise-once weight panel + CTA-pair kernel ("panel", the default for
    # M > 1024).  Same tolerances as test_awq_gemm_matches_fp32 and the residual test.  The
    # SiLU epilogue is checked against silu(x Wg) * (x Wu) in fp32 with the bf16 output
    # tolerance (it applies silu to the fp32 accumulators, one rounding at the end).
    import os, subprocess, sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if config == "panel":
        env = dict(os.environ, MES_GEMM_CONFIG="0", MES_GEMM_PANEL="1")
    else:
        env = dict(os.environ, MES_GEMM_CONFIG=config, MES_GEMM_PANEL="0")
    r = subprocess.run([sys.executable, "-c", _VARIANT_CHECK, root], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-3000:]


def test_awq_gemm_split_k_under_sm_reserve():
    # The overlapped tensor-parallel forward keeps SMs free for NCCL (mes_set_sm_reserve); the
    # split-K launch then sizes its clusters for the remaining SMs.  Same tolerance as
    # test_awq_gemm_matches_fp32; the reserve is restored whatever happens.
    try:
        _C.set_sm_reserve(64)
        for M, K, N in [(16, 2048, 1024), (200, 1024, 512), (64, 4096, 256)]:
            y, ref = _gemm_case(M, K, N, M % 2 == 0, seed=M + 7)
            err = (y - ref).abs().max().item()
            assert err <= 1e-2 * ref.abs().max().item() + 1e-3, (M, K, N, err)
    finally:
        _C.set_sm_reserve(0)
    assert _C.take_device_error() == 0


# ---------------------------------------------------------------- split-K over clusters
_SPLIT_CHECK = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import __graft_entry__; __graft_entry__.load_package()
from mes_b200 import _C
from oracle import awq as oawq
# Shapes of the one-tile-per-CTA kernel (M <= 64, or few 256-token tiles): 16/32/64/256-
# token tiles, ragged last tiles, K of 5 and 7 groups (uneven shares), bias, and all three
# epilogues.  Every result is computed twice and must repeat bit for bit.
for M, K, N, kind, bias in [(1, 640, 128, "bf16", True), (16, 896, 256, "res", False),
                            (33, 1024, 384, "silu", False), (64, 640, 256, "bf16", False),
                            (100, 896, 256, "res", True), (300, 1024, 512, "silu", False),
                            (256, 2048, 128, "bf16", True)]:
    qw, qz, sc = oawq.random_awq(K, N, seed=M + K)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16) if bias else None
    w = torch.from_numpy(oawq.bf16_bits_to_f32(oawq.dequant_bf16_bits(qw, qz, sc)))
    acc = x.float() @ w + (b.float() if b is not None else 0)
    dq, ds = torch.from_numpy(qz).cuda(), torch.from_numpy(sc).view(torch.int16).cuda()
    bd = None if b is None else b.cuda()
    outs = []
    for _ in range(2):
        if kind == "silu":
            qwi, qzi, sci = _C.interleave_gate_up(torch.from_numpy(qw).cuda(), dq, ds)
            got = _C.awq_gemm_silu(x.cuda(), _C.awq_repack(qwi), qzi, sci).float().cpu()
            ref = torch.nn.functional.silu(acc[:, : N // 2]) * acc[:, N // 2:]
            tol = 1e-2 * ref.abs().max().item() + 1e-3
        elif kind == "res":
            r0 = torch.randn(M, N, generator=torch.Generator().manual_seed(K))
            r = r0.cuda()
            _C.awq_gemm_residual(x.cuda(), _C.awq_repack(torch.from_numpy(qw).cuda()), dq, ds, r, bd)
            got, ref = r.cpu(), r0 + acc
            tol = 1e-4 * ref.abs().max().item() + 1e-4
        else:
            got = _C.awq_gemm(x.cuda(), _C.awq_repack(torch.from_numpy(qw).cuda()), dq, ds, bd).float().cpu()
            ref, tol = acc, 1e-2 * acc.abs().max().item() + 1e-3
        err = (got - ref).abs().max().item()
        assert err <= tol, (M, K, N, kind, err, tol)
        outs.append(got)
    assert torch.equal(outs[0], outs[1]), ("not deterministic", M, K, N, kind)
assert _C.take_device_error() == 0
print("ok")
"""


@pytest.mark.parametrize("split", ["1", "2", "3", "5", "8"])
def test_awq_gemm_split_k(split):
    # K split over clusters of `split` CTAs (MES_GEMM_SPLIT, read once per process, so each
    # value runs in a child process; capped by the K / 128 groups of the shape).  Same
    # tolerances as the unsplit tests; the cluster reduction adds the partial tiles in rank
    # order, so repeated calls agree bit for bit.
    import os, subprocess, sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, MES_GEMM_SPLIT=split)
    r = subprocess.run([sys.executable, "-c", _SPLIT_CHECK, root], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-3000:]


# ------------------------------------------------------------------ weight panel path
def _awq_case_dev(M, K, N, seed):
    qw, qz, sc = oawq.random_awq(K, N, seed=seed)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(DEV)
    return (x, torch.from_numpy(qw).to(DEV), torch.from_numpy(qz).to(DEV),
            torch.from_numpy(sc).view(torch.int16).to(DEV))


@pytest.mark.parametrize("M,K,N", [(1025, 1024, 512), (2000, 2048, 1024), (5000, 1024, 6144)])
def test_awq_gemm_panel_equals_fused(M, K, N):
    # The weight panel holds the same exactly-dequantised bf16 values the fused kernels
    # build in shared memory, and the residual epilogue runs the same CTA-pair MMAs on
    # them in the same k order in both paths: the fp32 sums must agree bit for bit.  The
    # bf16 and SiLU epilogues (single-CTA MMAs in the fused path) must agree within the
    # bf16 output tolerance.
    x, qw, qz, sc = _awq_case_dev(M, K, N, seed=M)
    qwm = _C.awq_repack(qw)
    assert _C.lib().mes_awq_gemm_workspace_size(M, N, K) == N * K * 2
    r0 = torch.randn(M, N, generator=torch.Generator().manual_seed(1)).to(DEV)
    outs = {}
    for panel in (True, False):
        _C.use_gemm_workspace = panel
        try:
            r = r0.clone()
            _C.awq_gemm_residual(x, qwm, qz, sc, r)
            y = _C.awq_gemm(x, qwm, qz, sc)
            qwi, qzi, sci = _C.interleave_gate_up(qw, qz, sc)
            z = _C.awq_gemm_silu(x, _C.awq_repack(qwi), qzi, sci)
            outs[panel] = (r, y, z)
        finally:
            _C.use_gemm_workspace = True
    # Panels prepared in one batched launch (as a decoder layer does) and passed in give the
    # same result as the per-call workspace.
    qwi, qzi, sci = _C.interleave_gate_up(qw, qz, sc)
    qwim = _C.awq_repack(qwi)
    pa = torch.empty(N, K, dtype=torch.bfloat16, device=DEV)
    pb = torch.empty(N, K, dtype=torch.bfloat16, device=DEV)
    _C.awq_panels([(qwm, qz, sc), (qwim, qzi, sci)], [pa, pb])
    w_ref = _C.awq_dequant(qwm, qz, sc)                  # W^T [N, K], the GEMM's arithmetic
    assert torch.equal(pa, w_ref)
    r = r0.clone()
    _C.awq_gemm_residual(x, qwm, qz, sc, r, panel=pa)
    y = _C.awq_gemm(x, qwm, qz, sc, panel=pa)
    z = _C.awq_gemm_silu(x, qwim, qzi, sci, panel=pb)
    assert _C.take_device_error() == 0
    assert torch.equal(r, outs[True][0]) and torch.equal(y, outs[True][1])
    assert torch.equal(z, outs[True][2])
    assert torch.equal(outs[True][0], outs[False][0])
    for a, b in zip(outs[True][1:], outs[False][1:]):
        a, b = a.float(), b.float()
        assert (a - b).abs().max().item() <= 1e-2 * b.abs().max().item()


@pytest.mark.parametrize("M,K,N", [(300, 1024, 512), (2000, 2048, 1024)])
def test_awq_gemm_residual_reduce_add_equals_register_path(M, K, N):
    # A 16-byte-aligned residual with rows a multiple of 4 floats apart is updated by TMA
    # reduce-adds in L2; any other layout by the epilogue's own read-modify-write.  Both add
    # acc + bias to R once in fp32, so the results must agree bit for bit.
    x, qw, qz, sc = _awq_case_dev(M, K, N, seed=M + 7)
    qwm = _C.awq_repack(qw)
    g = torch.Generator().manual_seed(M)
    r0 = torch.randn(M, N, generator=g).to(DEV)
    b = (0.1 * torch.randn(N, generator=g)).to(torch.bfloat16).to(DEV)
    aligned = r0.clone()
    _C.awq_gemm_residual(x, qwm, qz, sc, aligned, b)
    strided = torch.zeros(M, N + 1, device=DEV)[:, :N]   # rows N + 1 floats apart
    strided.copy_(r0)
    _C.awq_gemm_residual(x, qwm, qz, sc, strided, b)
    assert _C.take_device_error() == 0
    assert torch.equal(aligned, strided)
    w = _C.awq_dequant(qwm, qz, sc).float()              # W^T [N, K]
    want = r0 + (x.float() @ w.t() + b.float())
    assert (aligned - want).abs().max().item() <= 1e-4 * want.abs().max().item()


def test_awq_gemm_workspace_size_rules():
    # The panel path serves batches of more than 1024 tokens whose N is a multiple of 256;
    # everything else reports 0 (the fused kernels need no workspace).
    size = _C.lib().mes_awq_gemm_workspace_size
    assert size(256, 1024, 1024) == 0
    assert size(1024, 1024, 1024) == 0              # the dequantising pair kernel
    assert size(1025, 1024, 1024) == 1024 * 1024 * 2
    assert size(20000, 384, 1024) == 0
    assert size(20000, 6144, 1024) == 6144 * 1024 * 2


def test_awq_gemm_rows_independent_of_batch_and_sm_reserve():
    # For more than 256 tokens a row's result must not depend on the rest of the batch or on
    # how many SMs the persistent kernels may use: the tensor-parallel overlap runs
    # micro-batches under an SM reserve and must equal the unsplit forward bit for bit, and
    # a padded CUDA-graph batch must give its real rows exactly.  Shapes of the 0.6B model
    # at TP2 (QKV N = 2048, gate_up N = 3072, o/down N = 1024).
    for K, N, epi in [(1024, 2048, "bf16"), (1024, 3072, "silu"), (1536, 1024, "residual")]:
        x, qw, qz, sc = _awq_case_dev(5000, K, N, seed=N)
        if epi == "silu":
            qw, qz, sc = _C.interleave_gate_up(qw, qz, sc)
        qwm = _C.awq_repack(qw)

        def run(rows, reserve):
            _C.set_sm_reserve(reserve)
            try:
                xs = x[:rows].contiguous()
                if epi == "residual":
                    r = torch.zeros(rows, N, device=DEV)
                    return _C.awq_gemm_residual(xs, qwm, qz, sc, r)
                if epi == "silu":
                    return _C.awq_gemm_silu(xs, qwm, qz, sc)
                return _C.awq_gemm(xs, qwm, qz, sc)
            finally:
                _C.set_sm_reserve(0)

        full = run(5000, 0)
        # 1025 and more rows run on a weight panel, 257-1024 on the dequantising pair
        # kernel: the same MMAs in the same k order.
        for rows, reserve in [(5000, 16), (3000, 16), (2000, 0), (4096, 24), (1025, 0),
                              (1024, 0), (777, 0), (300, 16)]:
            assert torch.equal(run(rows, reserve), full[:rows]), (K, N, epi, rows, reserve)
    assert _C.take_device_error() == 0
