"""Seeded synthetic models and batches for the benchmark workloads.

There are no checkpoints or datasets on the benchmark hosts, so models are built from
their published architecture numbers with seeded random weights and batches are seeded
random token ids.  Weight tensors use checkpoint (HF) names, so they load through the
ordinary ``load_weights`` path.

* ``dense_weights``: fp32 ``normal(0, 0.02)`` for every matrix, ones for norms.
* ``awq_weights``: AWQ int4 tensors for every linear (codes and zero-points uniform in
  [0, 15], fp16 scales uniform in [0.002, 0.02], group 128) and bf16 ``normal(0, 0.02)``
  embeddings / biases; norms are ones (or ``1 + norm_noise * normal``).
* batches: ``packed_batch(lengths)`` -> ids uniform in [0, vocab), positions
  ``0..len-1`` per sequence, last-token indices (``core/tokenizer_manager.py:151-166``).
"""
from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import torch

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
GROUP = 128


# ------------------------------------------------------------------------ architectures
def _cfg(arch: str, arch_kw: dict, overrides: dict):
    base = dict(rms_norm_eps=1e-6, hidden_act="silu", max_position_embeddings=40960,
                rope_theta=1000000.0, attention_bias=False, architectures=[arch],
                rope_scaling=None)
    base.update(arch_kw)
    base.update(overrides)
    return SimpleNamespace(**base)


def qwen3_0_6b(**kw):
    """Qwen3-Embedding-0.6B architecture."""
    return _cfg("Qwen3ForCausalLM", dict(vocab_size=151669, hidden_size=1024, num_hidden_layers=28,
                num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                intermediate_size=3072), kw)


def qwen3_4b(**kw):
    """Qwen3-Embedding-4B architecture (projection shapes of the GEMM microbenchmark)."""
    return _cfg("Qwen3ForCausalLM", dict(vocab_size=151669, hidden_size=2560, num_hidden_layers=36,
                num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                intermediate_size=9728), kw)


def qwen3_8b(**kw):
    """Qwen3-Embedding-8B architecture."""
    return _cfg("Qwen3ForCausalLM", dict(vocab_size=151669, hidden_size=4096, num_hidden_layers=36,
                num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                intermediate_size=12288), kw)


def qwen2_1_5b(**kw):
    """Qwen2-1.5B architecture (QKV bias, no q/k norm)."""
    return _cfg("Qwen2ForCausalLM", dict(vocab_size=151936, hidden_size=1536, num_hidden_layers=28,
                num_attention_heads=12, num_key_value_heads=2, head_dim=128,
                intermediate_size=8960), kw)


def is_qwen2(cfg) -> bool:
    return cfg.architectures[0] == "Qwen2ForCausalLM"


def linear_shapes(cfg) -> dict:
    """HF projection name -> (K, N) = (in_features, out_features)."""
    H, D = cfg.hidden_size, getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    Hq, Hkv, I = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.intermediate_size
    return {
        "self_attn.q_proj": (H, Hq * D), "self_attn.k_proj": (H, Hkv * D),
        "self_attn.v_proj": (H, Hkv * D), "self_attn.o_proj": (Hq * D, H),
        "mlp.gate_proj": (H, I), "mlp.up_proj": (H, I), "mlp.down_proj": (I, H),
    }


# ------------------------------------------------------------------------ AWQ packing
def pack_awq(codes: torch.Tensor) -> torch.Tensor:
    """uint8 codes ``[R, C]`` -> AWQ-packed int32 ``[R, C/8]`` (nibble i = column
    ``8j + AWQ_ORDER[i]``)."""
    R, C = codes.shape
    q = codes.view(R, C // 8, 8).to(torch.int64)
    out = torch.zeros(R, C // 8, dtype=torch.int64, device=codes.device)
    for i, src in enumerate(AWQ_ORDER):
        out |= (q[:, :, src] & 0xF) << (4 * i)
    out = torch.where(out >= 2 ** 31, out - 2 ** 32, out)
    return out.to(torch.int32)


def random_awq(K: int, N: int, gen: torch.Generator, device="cpu",
               scale_lo: float = 0.002, scale_hi: float = 0.02, zero_lo: int = 0,
               zero_hi: int = 15):
    q = torch.randint(0, 16, (K, N), generator=gen, device=device, dtype=torch.uint8)
    z = torch.randint(zero_lo, zero_hi + 1, (K // GROUP, N), generator=gen, device=device,
                      dtype=torch.uint8)
    s = torch.rand((K // GROUP, N), generator=gen, device=device)
    s = (s * (scale_hi - scale_lo) + scale_lo).to(torch.float16)
    return pack_awq(q), pack_awq(z), s


def quantize_awq(w: torch.Tensor, group: int = GROUP):
    """Round-to-nearest asymmetric 4-bit group quantisation of a dense ``[out, in]`` weight
    into AWQ checkpoint tensors (qweight ``[in, out/8]``, qzeros ``[in/G, out/8]``, fp16
    scales ``[in/G, out]``): per group of ``group`` input features, s = (max - min) / 15,
    z = clamp(round(-min / s), 0, 15), q = clamp(round(w / s) + z, 0, 15)."""
    wt = w.t().float()                                   # [K, N]
    K, N = wt.shape
    g = wt.reshape(K // group, group, N)
    lo, hi = g.amin(1), g.amax(1)
    s = ((hi - lo).clamp(min=1e-5) / 15).to(torch.float16)
    sf = s.float()
    z = (-torch.round(lo / sf)).clamp(0, 15)
    q = (torch.round(g / sf[:, None, :]) + z[:, None, :]).clamp(0, 15)
    return (pack_awq(q.reshape(K, N).to(torch.uint8)), pack_awq(z.to(torch.uint8)), s)


def quantize_dense_checkpoint(dense: dict) -> dict:
    """Dense checkpoint-named weights -> AWQ checkpoint (linears quantised, embeddings and
    biases in bf16, norms copied)."""
    out = {}
    for name, t in dense.items():
        if name.endswith("_proj.weight"):
            base = name[: -len(".weight")]
            out[base + ".qweight"], out[base + ".qzeros"], out[base + ".scales"] = quantize_awq(t)
        elif name.endswith(".bias") or name == "embed_tokens.weight":
            out[name] = t.to(torch.bfloat16)
        else:
            out[name] = t.to(torch.bfloat16)
    return out


def _gen(seed: int, device) -> torch.Generator:
    return torch.Generator(device=torch.device(device)).manual_seed(seed)


def awq_weights(cfg, seed: int = 0, device="cpu", num_layers: int | None = None,
                norm_noise: float = 0.0, zero_range: tuple[int, int] = (0, 15)) -> dict:
    """Checkpoint-named AWQ model tensors, generated in a fixed order from ``seed``.
    ``zero_range`` bounds the zero-point codes (the benchmark configs use [0, 15];
    checkpoints produced by AWQ calibration sit near the midpoint, e.g. [7, 8])."""
    gen = _gen(seed, device)
    L = cfg.num_hidden_layers if num_layers is None else num_layers
    H = cfg.hidden_size
    D = getattr(cfg, "head_dim", None) or H // cfg.num_attention_heads
    qwen2 = is_qwen2(cfg)
    out = {}

    def normal(*shape, std=0.02):
        return (torch.randn(*shape, generator=gen, device=device) * std).to(torch.bfloat16)

    def norm(n):
        if norm_noise == 0.0:
            return torch.ones(n, dtype=torch.bfloat16, device=device)
        return (1.0 + norm_noise * torch.randn(n, generator=gen, device=device)).to(torch.bfloat16)

    out["embed_tokens.weight"] = normal(cfg.vocab_size, H)
    for i in range(L):
        p = f"layers.{i}."
        out[p + "input_layernorm.weight"] = norm(H)
        for name, (K, N) in linear_shapes(cfg).items():
            qw, qz, sc = random_awq(K, N, gen, device, zero_lo=zero_range[0],
                                    zero_hi=zero_range[1])
            out[p + name + ".qweight"], out[p + name + ".qzeros"], out[p + name + ".scales"] = qw, qz, sc
            if qwen2 and name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
                out[p + name + ".bias"] = normal(N)
        if not qwen2:
            out[p + "self_attn.q_norm.weight"] = norm(D)
            out[p + "self_attn.k_norm.weight"] = norm(D)
        out[p + "post_attention_layernorm.weight"] = norm(H)
    out["norm.weight"] = norm(H)
    return out


def dense_weights(cfg, seed: int = 0, num_layers: int | None = None, std: float = 0.02) -> dict:
    """Checkpoint-named dense fp32 tensors (``[out, in]``), generated in a fixed order."""
    gen = _gen(seed, "cpu")
    L = cfg.num_hidden_layers if num_layers is None else num_layers
    H = cfg.hidden_size
    D = getattr(cfg, "head_dim", None) or H // cfg.num_attention_heads
    qwen2 = is_qwen2(cfg)
    out = {"embed_tokens.weight": torch.randn(cfg.vocab_size, H, generator=gen) * std}
    for i in range(L):
        p = f"layers.{i}."
        out[p + "input_layernorm.weight"] = torch.ones(H)
        for name, (K, N) in linear_shapes(cfg).items():
            out[p + name + ".weight"] = torch.randn(N, K, generator=gen) * std
            if qwen2 and name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"):
                out[p + name + ".bias"] = torch.randn(N, generator=gen) * std
        if not qwen2:
            out[p + "self_attn.q_norm.weight"] = torch.ones(D)
            out[p + "self_attn.k_norm.weight"] = torch.ones(D)
        out[p + "post_attention_layernorm.weight"] = torch.ones(H)
    out["norm.weight"] = torch.ones(H)
    return out


# ------------------------------------------------------------------------ batches
def packed_batch(lengths, vocab: int, seed: int = 1):
    """(input_ids int64 [T], positions int64 [T], last_token_indices int64 [B]) as numpy."""
    lengths = [int(n) for n in lengths]
    rng = np.random.default_rng(seed)
    T = sum(lengths)
    ids = rng.integers(0, vocab, size=T, dtype=np.int64)
    positions = np.concatenate([np.arange(n, dtype=np.int64) for n in lengths]) if T else \
        np.zeros(0, dtype=np.int64)
    last = np.cumsum(lengths, dtype=np.int64) - 1
    return ids, positions, last


def lengths_uniform(n: int, lo: int, hi: int, seed: int = 1) -> list[int]:
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=n).tolist()


def lengths_log_uniform(total: int, lo: int, hi: int, seed: int = 1) -> list[int]:
    """floor(exp(U(ln lo, ln hi))) until the sum reaches ``total``; the last is trimmed."""
    rng = np.random.default_rng(seed)
    out, s = [], 0
    while s < total:
        n = int(math.floor(math.exp(rng.uniform(math.log(lo), math.log(hi)))))
        n = min(n, total - s)
        out.append(n)
        s += n
    return out
