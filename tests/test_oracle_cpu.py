"""CPU tests: the oracle against the reference's golden fixtures, the AWQ format against
vLLM's packer, and the C-ABI library's exports (no GPU work)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from mes_b200 import _C, synthetic
from oracle import awq as oawq
from oracle import model as omodel
from oracle import ops

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


# ------------------------------------------------------------------------ AWQ format
def test_awq_pack_order_matches_vllm():
    f = golden("awq_pack_vllm.npz")
    codes, packed = f["codes"], f["packed"]
    assert np.array_equal(oawq.awq_pack(codes), packed)
    assert np.array_equal(oawq.awq_unpack(packed), codes)
    assert np.array_equal(synthetic.pack_awq(torch.from_numpy(codes)).numpy(), packed)


def test_kernel_layout_repack_is_lossless():
    qw, _, _ = oawq.random_awq(512, 256, seed=3)
    mes = oawq.mes_repack(qw)
    assert mes.shape == (512 // 8, 256)
    assert np.array_equal(oawq.mes_unpack(mes), oawq.awq_unpack(qw))
    # word (b, n) holds k = 8b + order[i] at nibble i
    q = oawq.awq_unpack(qw)
    w = mes.view(np.uint32)
    for i, k in enumerate(oawq.AWQ_ORDER):
        assert np.array_equal((w[3] >> (4 * i)) & 0xF, q[24 + k])


def test_dequant_is_exact_and_rounds_once():
    qw, qz, sc = oawq.random_awq(256, 128, seed=4)
    got = oawq.dequant_fp32(qw, qz, sc)
    q = oawq.awq_unpack(qw).astype(np.float64)
    z = np.repeat(oawq.awq_unpack(qz).astype(np.float64), 128, 0)
    s = np.repeat(sc.astype(np.float64), 128, 0)
    assert np.array_equal(got.astype(np.float64), (q - z) * s)   # exact in fp32
    bits = oawq.dequant_bf16_bits(qw, qz, sc)
    want = torch.from_numpy(got).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, want)                               # RNE, as torch rounds


def test_bf16_rounding_ties_to_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8, 3.0e38, 1e-40, 0.0, -0.0],
                 dtype=np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oawq.f32_to_bf16_bits(x), want)


def test_rtn_quantiser_reconstructs_dense_weights():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(256, 512, generator=g) * 0.02
    qw, qz, sc = synthetic.quantize_awq(w)
    rec = oawq.dequant_fp32(qw.numpy(), qz.numpy(), sc.numpy()).T
    step = sc.float().numpy().max()
    assert np.abs(rec - w.numpy()).max() <= 0.51 * step + 1e-6


# ------------------------------------------------------------------------ per-op parity
def test_ops_match_reference_layers():
    f = golden("ref_ops.npz")
    bf = torch.bfloat16
    # bf16: the reference's deployment dtype; the oracle performs the same roundings.
    x, r, w = (torch.from_numpy(f[k]).to(bf) for k in ("rms_x_bf16", "rms_r_bf16", "rms_w_bf16"))
    assert torch.equal(ops.rms_norm(x, w, 1e-6).float(), torch.from_numpy(f["rms_y_bf16"]))
    y, res = ops.add_rms_norm(x, r, w, 1e-6)
    assert torch.equal(y.float(), torch.from_numpy(f["addrms_y_bf16"]))
    assert torch.equal(res.float(), torch.from_numpy(f["addrms_res_bf16"]))
    g = torch.from_numpy(f["silu_x_bf16"]).to(bf)
    assert torch.equal(ops.silu_and_mul(g).float(), torch.from_numpy(f["silu_y_bf16"]))
    # fp32 (the reference's fp32 add_rms returns an aliased residual; its output is right)
    x, r, w = (torch.from_numpy(f[k]) for k in ("rms_x_fp32", "rms_r_fp32", "rms_w_fp32"))
    assert torch.allclose(ops.rms_norm(x, w, 1e-6), torch.from_numpy(f["rms_y_fp32"]), atol=1e-6)
    y, _ = ops.add_rms_norm(x, r, w, 1e-6)
    assert torch.allclose(y, torch.from_numpy(f["addrms_y_fp32"]), atol=1e-6)
    assert torch.allclose(ops.silu_and_mul(torch.from_numpy(f["silu_x_fp32"])),
                          torch.from_numpy(f["silu_y_fp32"]), atol=1e-6)


def test_rope_matches_reference():
    f = golden("ref_ops.npz")
    pos = torch.from_numpy(f["rope_pos"])
    q, k = torch.from_numpy(f["rope_q"]), torch.from_numpy(f["rope_k"])
    cache = ops.rope_cos_sin_cache(128, 4096, 1e6)
    assert torch.allclose(ops.apply_rope(q, pos, cache, 128), torch.from_numpy(f["rope_q_out"]), atol=1e-6)
    assert torch.allclose(ops.apply_rope(k, pos, cache, 128), torch.from_numpy(f["rope_k_out"]), atol=1e-6)
    bf = torch.bfloat16
    qb = ops.apply_rope(q.to(bf), pos, cache.to(bf), 128).float()
    assert torch.equal(qb, torch.from_numpy(f["rope_q_out_bf16"]))


def test_attention_backend_matches_reference():
    f = golden("ref_ops.npz")
    pos = torch.from_numpy(f["rope_pos"])
    cu = ops.cu_seqlens_from_positions(pos)
    assert cu.tolist() == [0, 20, 53, 56]
    out = ops.varlen_causal_attention(*(torch.from_numpy(f[k]) for k in ("attn_q", "attn_k", "attn_v")),
                                      cu, 8, 2, 128)
    assert torch.allclose(out, torch.from_numpy(f["attn_out"]), atol=1e-5)


# ------------------------------------------------------------------------ model parity
def _cos(a, b):
    return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))


@pytest.mark.parametrize("fixture,cfg,qk_norm", [
    ("ref_qwen3_c1.npz", synthetic.qwen3_0_6b(max_position_embeddings=32768), True),
    ("ref_qwen2_small.npz", synthetic.qwen2_1_5b(num_hidden_layers=2, max_position_embeddings=32768), False),
])
def test_oracle_model_matches_reference_forward(fixture, cfg, qk_norm):
    f = golden(fixture)
    w = synthetic.dense_weights(cfg, seed=int(f["weight_seed"]))
    emb = omodel.embed(cfg, w, torch.from_numpy(f["ids"]), torch.from_numpy(f["positions"]),
                       torch.from_numpy(f["last"]), qk_norm=qk_norm).numpy()
    # Same fp32 arithmetic as the reference's (alias-fixed) fp32 path; differences come
    # only from summation order inside matmul / SDPA.
    assert np.abs(emb - f["emb_fp32"]).max() < 1e-5
    assert _cos(emb, f["emb_fp32"]).min() > 0.999999
    # The reference's deployment dtype (bf16) against fp32, and its fp32 aliasing defect.
    assert _cos(f["emb_bf16"], f["emb_fp32"]).min() > 0.999
    assert _cos(f["emb_fp32_as_is"], f["emb_fp32"]).min() < 0.99


# ------------------------------------------------------------------------ C ABI
def _header_functions():
    text = open(os.path.join(ROOT, "include", "mes_b200.h")).read()
    return sorted(set(re.findall(r"^(?:int|int64_t|const char\*)\s+(mes_\w+)\(", text, re.M)))


def test_library_loads_and_exports_every_header_symbol():
    lib = _C.lib()
    names = _header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
        assert n in _C.SIGNATURES, n
    assert lib.mes_version() >= 100
    assert _C.status_string(1) == "invalid argument or unsupported shape"


def test_binding_signatures_mirror_the_header():
    """Every prototype of the header has the ctypes signature ``_C`` declares: the same
    return type and, argument by argument, a pointer, int64, int or float."""
    import ctypes
    text = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", "mes_b200.h")).read(),
                  flags=re.S)
    protos = re.findall(r"^(int|int64_t|const char\*)\s+(mes_\w+)\(([^;]*?)\);", text, re.M | re.S)
    assert len(protos) == len(_header_functions())
    ret_kind = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "const char*": ctypes.c_char_p}
    arg_kind = {ctypes.c_void_p: "ptr", ctypes.c_int64: "int64_t", ctypes.c_int: "int",
                ctypes.c_float: "float"}
    for ret, name, params in protos:
        want = []
        for prm in params.split(","):
            prm = " ".join(prm.split())
            if prm and prm != "void":
                want.append("ptr" if "*" in prm else prm.rsplit(" ", 1)[0])
        res, args = _C.SIGNATURES[name]
        assert res is ret_kind[ret], name
        assert [arg_kind.get(a, "ptr") for a in args] == want, name


def test_host_argument_checks_reject_without_gpu_work():
    lib = _C.lib()
    # N not a multiple of 128 -> MES_ERR_INVALID before any CUDA call
    assert lib.mes_awq_gemm(None, 64, None, None, None, None, None, 100, 16, 100, 64, 128, None) == 1
    assert lib.mes_varlen_workspace_size(-1) == -1
    assert lib.mes_varlen_workspace_size(1000) >= 4 * 1001 + 8 * 1000
    # GEMM weight-panel workspace: only batches of more than 1024 tokens with N a multiple of
    # the 256-feature pair tile use one; an unknown epilogue is rejected on the host.
    assert lib.mes_awq_gemm_workspace_size(256, 1024, 1024) == 0
    assert lib.mes_awq_gemm_workspace_size(1024, 1024, 1024) == 0
    assert lib.mes_awq_gemm_workspace_size(1025, 1024, 1024) == 1024 * 1024 * 2
    assert lib.mes_awq_gemm_workspace_size(20000, 384, 1024) == 0
    assert lib.mes_awq_gemm_ws(3, None, 64, None, None, None, None, None, 64, 16, 128, 64, 128,
                               None, 0, None) == 1
    assert lib.mes_awq_gemm_on_panel(0, None, 1024, None, None, None, 1024, 1024, 1024, 1024,
                                     None) == 1     # M <= 1024: no panel path
    assert lib.mes_awq_panels(0, None, None, None, None, None, None, None) == 1
    assert lib.mes_wait_probe(0, 0, None) == 1             # limit out of range
    assert lib.mes_wait_probe(1_000_000_000, 0, None) == 1
    # Pointers that do not start on the boundary their elements (or TMA) need are refused
    # with MES_ERR_ALIGN before anything is launched (the addresses are never dereferenced).
    a, odd4, odd2 = 0x10000, 0x10004, 0x10002
    assert lib.mes_embedding(odd4, 4, a, 10, 8, a, None) == 2                  # ids (i64)
    assert lib.mes_embedding_f32(odd4, 4, a, 10, 8, a, None) == 2
    assert lib.mes_qknorm_rope(a, 256, odd4, a, 1, 64, None, None, 4, 1, 1, 128, 1e-6, 0,
                               None) == 2                                         # positions
    assert lib.mes_last_token_l2(a, 4, 8, odd4, 1, a, None) == 2                 # indices
    assert lib.mes_varlen_schedule(odd4, 4, a, None) == 2                         # positions
    assert lib.mes_awq_repack(odd2, 128, 8, a, None) == 2                         # i32 words
    assert lib.mes_awq_dequant(a, odd2, a, 128, 8, 128, a, None) == 2
    assert lib.mes_awq_dequant(a, a, a + 1, 128, 8, 128, a, None) == 2           # f16 scales
    vp = ctypes.c_void_p
    i64 = ctypes.c_int64
    assert lib.mes_awq_panels(1, (vp * 1)(a), (vp * 1)(odd2), (vp * 1)(a), (i64 * 1)(128),
                              (i64 * 1)(8), (vp * 1)(a), None) == 2
    for qz, sc, b in ((odd4, a, None), (a, odd4, None), (a, a, a + 1)):         # TMA-read / bias
        assert lib.mes_awq_gemm(a, 128, a, qz, sc, b, a, 128, 16, 128, 128, 128, None) == 2
    assert lib.mes_awq_gemm_on_panel(0, a, 1024, a, a + 1, a, 1024, 2048, 1024, 1024, None) == 2


def test_cpu_tensors_raise_instead_of_falling_back():
    with pytest.raises(_C.MesError):
        _C.silu_mul(torch.zeros(4, 16, dtype=torch.bfloat16))


def test_last_token_pool_matches_oracle_post_process():
    """``last_token_pool`` per sequence of a packed batch, then the L2 normalisation, is the
    oracle's post-process (``ultils/pool.py:4-9``, ``core/gpu_worker.py:252-261``)."""
    from mes_b200.ultils.pool import last_token_pool
    g = torch.Generator().manual_seed(7)
    lengths = [5, 1, 17, 3]
    hidden = torch.randn(sum(lengths), 64, generator=g).to(torch.bfloat16)
    hidden[5 + 1 - 1] = 0          # a zero row: normalised by max(||x||, 1e-12)
    starts = np.cumsum([0] + lengths[:-1])
    pooled = torch.stack([last_token_pool(hidden[s:s + n], n) for s, n in zip(starts, lengths)])
    got = torch.nn.functional.normalize(pooled.float(), p=2, dim=1)
    want = ops.last_token_l2(hidden, starts + np.array(lengths) - 1)
    assert torch.equal(got, want)
    assert not torch.isnan(got).any()
