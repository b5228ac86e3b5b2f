"""Qwen3 / Qwen2 decoder forward restated on the CPU (oracle only).

Follows ``models/qwen3.py:81-166`` and ``models/qwen2.py:81-192`` of the reference:

* embed -> for each layer: (add+)RMSNorm -> QKV projection (+bias for Qwen2) ->
  per-head q/k RMSNorm (Qwen3 only, ``qwen3.py:82-88``) -> NeoX RoPE -> varlen causal
  GQA attention -> o_proj (+all-reduce at tp>1) -> add+RMSNorm -> gate_up -> SiLU-and-mul
  -> down_proj (+all-reduce at tp>1) -> final add+RMSNorm (``qwen3.py:165``).
* Weights use the checkpoint (HF) names, dense ``[out, in]``.  ``awq_dense_weights``
  turns AWQ tensors into the "fp32 dequantised reference" weights.
* Tensor parallelism follows ``layers/linear.py``: column-parallel q/k/v and gate/up
  shards hold ``1/tp`` of the heads / intermediate features, row-parallel o/down hold
  ``1/tp`` of the input features and their outputs are summed with ``all_reduce``
  (``linear.py:176-180``).  The embedding is replicated instead of vocab-sharded; the
  result is identical because the reference's masked shards sum to exactly one row
  (``embed_head.py:43-52``).
"""
from __future__ import annotations

import numpy as np
import torch

from . import awq as awq_ref
from . import ops

PROJS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
COLUMN_PROJS = ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")


def arch(cfg) -> dict:
    """Architecture numbers read from an HF-style config object."""
    H = cfg.hidden_size
    Hq = cfg.num_attention_heads
    D = getattr(cfg, "head_dim", None) or H // Hq
    return dict(
        vocab=cfg.vocab_size, hidden=H, heads=Hq, kv_heads=cfg.num_key_value_heads,
        head_dim=D, inter=cfg.intermediate_size, layers=cfg.num_hidden_layers,
        eps=cfg.rms_norm_eps,
        theta=float(getattr(cfg, "rope_theta", None) or 1000000.0),
        max_pos=cfg.max_position_embeddings,
    )


def awq_dense_weights(awq_weights: dict, group_size: int = 128) -> dict:
    """Replace every ``<proj>.qweight/qzeros/scales`` triple by the exact fp32 dequantised
    dense ``<proj>.weight`` ``[N, K]`` (AWQ stores ``[K, N]``); other tensors are copied."""
    out = {}
    for name, t in awq_weights.items():
        if name.endswith(".qweight"):
            base = name[: -len(".qweight")]
            w = awq_ref.dequant_fp32(np.asarray(t), np.asarray(awq_weights[base + ".qzeros"]),
                                     np.asarray(awq_weights[base + ".scales"]), group_size)
            out[base + ".weight"] = torch.from_numpy(np.ascontiguousarray(w.T))
        elif name.endswith(".qzeros") or name.endswith(".scales"):
            continue
        else:
            out[name] = torch.as_tensor(t).to(torch.float32)
    return out


def shard_dense(weights: dict, cfg, rank: int, world: int) -> dict:
    """Per-rank shard of dense HF-named weights, as ``layers/linear.py`` splits them."""
    a = arch(cfg)
    out = {}
    for name, t in weights.items():
        parts = name.split(".")
        proj = parts[-2] if len(parts) >= 2 else ""
        if proj in COLUMN_PROJS:
            out[name] = t.chunk(world, 0)[rank].contiguous()
        elif proj in ("o_proj", "down_proj") and parts[-1] == "weight":
            out[name] = t.chunk(world, 1)[rank].contiguous()
        elif proj in ("o_proj", "down_proj") and parts[-1] == "bias":
            out[name] = t if rank == 0 else torch.zeros_like(t)
        else:
            out[name] = t
    assert a["heads"] % world == 0 and a["kv_heads"] % world == 0
    return out


@torch.no_grad()
def forward(cfg, weights: dict, input_ids: torch.Tensor, positions: torch.Tensor,
            qk_norm: bool = True, dtype: torch.dtype = torch.float32,
            world: int = 1, group=None, num_layers: int | None = None) -> torch.Tensor:
    """Hidden states ``[T, H]`` of the last layer's final norm (``qwen3.py:156-166``).

    ``weights`` are this rank's shards (see :func:`shard_dense`); ``qk_norm`` selects
    Qwen3 (True) or Qwen2 (False) attention.  At ``world > 1`` the o/down outputs are
    summed over ``group`` with ``torch.distributed.all_reduce``.
    """
    import torch.distributed as dist

    a = arch(cfg)
    L = a["layers"] if num_layers is None else num_layers
    D, eps = a["head_dim"], a["eps"]
    hq, hkv = a["heads"] // world, a["kv_heads"] // world
    W = {k: v.to(dtype) for k, v in weights.items()}
    cache = ops.rope_cos_sin_cache(D, a["max_pos"], a["theta"]).to(dtype)

    def lin(x, prefix):
        y = x @ W[prefix + ".weight"].t()
        b = W.get(prefix + ".bias")
        return y if b is None else y + b

    def allreduce(y):
        if world > 1:
            dist.all_reduce(y, group=group)
        return y

    cu = ops.cu_seqlens_from_positions(positions)
    h = ops.embedding(input_ids, W["embed_tokens.weight"])
    residual = None
    for i in range(L):
        p = f"layers.{i}."
        if residual is None:
            residual = h
            x = ops.rms_norm(h, W[p + "input_layernorm.weight"], eps)
        else:
            x, residual = ops.add_rms_norm(h, residual, W[p + "input_layernorm.weight"], eps)
        q = lin(x, p + "self_attn.q_proj")
        k = lin(x, p + "self_attn.k_proj")
        v = lin(x, p + "self_attn.v_proj")
        T = q.shape[0]
        if qk_norm:
            q = ops.rms_norm(q.view(T, hq, D), W[p + "self_attn.q_norm.weight"], eps).view(T, -1)
            k = ops.rms_norm(k.view(T, hkv, D), W[p + "self_attn.k_norm.weight"], eps).view(T, -1)
        q = ops.apply_rope(q, positions, cache, D)
        k = ops.apply_rope(k, positions, cache, D)
        o = ops.varlen_causal_attention(q, k, v, cu, hq, hkv, D)
        h = allreduce(lin(o, p + "self_attn.o_proj"))
        x, residual = ops.add_rms_norm(h, residual, W[p + "post_attention_layernorm.weight"], eps)
        gu = torch.cat([lin(x, p + "mlp.gate_proj"), lin(x, p + "mlp.up_proj")], dim=-1)
        h = allreduce(lin(ops.silu_and_mul(gu), p + "mlp.down_proj"))
    out, _ = ops.add_rms_norm(h, residual, W["norm.weight"], eps)
    return out


def embed(cfg, weights, input_ids, positions, last_token_indices, **kw) -> torch.Tensor:
    """Forward + last-token pooling + L2 normalisation -> fp32 ``[B, H]``."""
    return ops.last_token_l2(forward(cfg, weights, input_ids, positions, **kw),
                             last_token_indices)
