"""Per-op restatements of the reference's layer arithmetic on the CPU (oracle only).

Every function takes and returns torch CPU tensors and computes in the dtype it is given
(fp32 for the parity oracle), following the cited reference line by line, except that
in-place aliasing defects of the reference's fp32 path are not reproduced: the reference
``RMSNorm`` mutates its input when the input is already fp32 (``layers/layernorm.py:23-25``
and ``:37-39``), which corrupts the residual stream in fp32 only.  Here every op is out
of place, which equals the reference's behaviour in its deployment dtype (bf16).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``RMSNorm.rms_forward`` (layers/layernorm.py:18-27): fp32 statistics, round to the
    input dtype, then multiply by the weight."""
    orig = x.dtype
    xf = x.to(torch.float32)
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    y = xf * torch.rsqrt(var + eps)
    return y.to(orig) * weight.to(orig)


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                 eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """``RMSNorm.add_rms_forward`` (layers/layernorm.py:30-41): the fp32 sum is both the
    new residual (rounded to the input dtype) and the input of the normalisation."""
    orig = x.dtype
    s = x.to(torch.float32) + residual.to(torch.float32)
    new_residual = s.to(orig)
    var = s.pow(2).mean(dim=-1, keepdim=True)
    y = (s * torch.rsqrt(var + eps)).to(orig) * weight.to(orig)
    return y, new_residual


def rope_cos_sin_cache(head_size: int, max_position: int, base: float) -> torch.Tensor:
    """``RotaryEmbedding.__init__`` (layers/rotary_embedding.py:29-37): fp32
    ``[max_position, head_size]`` = cat(cos, sin) of ``t * base^(-2i/d)``."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_size, 2, dtype=torch.float) / head_size))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cache: torch.Tensor,
               head_size: int) -> torch.Tensor:
    """``RotaryEmbedding.forward`` + ``apply_rotary_emb`` (layers/rotary_embedding.py:6-16,
    39-55): NeoX rotate-half on ``[T, heads*head_size]``, math in fp32 with the cache's
    cos/sin values, result rounded to the input dtype."""
    T = positions.shape[0]
    cos, sin = cache[positions].chunk(2, dim=-1)
    cos = cos.unsqueeze(-2).to(torch.float32)
    sin = sin.unsqueeze(-2).to(torch.float32)
    xs = x.reshape(T, -1, head_size)
    x1, x2 = torch.chunk(xs.to(torch.float32), 2, dim=-1)
    y = torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)
    return y.to(x.dtype).reshape(x.shape)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """``SiluAndMul.forward`` (layers/activation.py:12-14)."""
    g, u = x.chunk(2, -1)
    return F.silu(g) * u


def cu_seqlens_from_positions(positions: torch.Tensor) -> torch.Tensor:
    """Sequence boundaries where ``positions[i] != positions[i-1] + 1``
    (layers/attention/flashattention.py:26-34)."""
    bounds = [0]
    if len(positions) > 1:
        jumps = (positions[1:] != positions[:-1] + 1).nonzero(as_tuple=True)[0]
        bounds.extend((jumps + 1).tolist())
    bounds.append(len(positions))
    return torch.tensor(bounds, dtype=torch.int64)


def varlen_causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            cu_seqlens: torch.Tensor, num_heads: int, num_kv_heads: int,
                            head_dim: int, scale: float | None = None) -> torch.Tensor:
    """Per-sequence causal GQA softmax attention, the contract of
    ``flash_attn_varlen_func(causal=True)`` as called at
    layers/attention/flashattention.py:38-45 (query head ``h`` reads KV head
    ``h // (num_heads / num_kv_heads)``).  Inputs ``[T, heads*head_dim]``."""
    if scale is None:
        scale = head_dim ** -0.5
    T = q.shape[0]
    qh = q.reshape(T, num_heads, head_dim).to(torch.float32)
    kh = k.reshape(T, num_kv_heads, head_dim).to(torch.float32)
    vh = v.reshape(T, num_kv_heads, head_dim).to(torch.float32)
    rep = num_heads // num_kv_heads
    out = torch.empty(T, num_heads, head_dim, dtype=torch.float32)
    cu = cu_seqlens.tolist()
    for s, e in zip(cu[:-1], cu[1:]):
        if e <= s:
            continue
        qq = qh[s:e].transpose(0, 1)                                  # [H, L, D]
        kk = kh[s:e].repeat_interleave(rep, dim=1).transpose(0, 1)
        vv = vh[s:e].repeat_interleave(rep, dim=1).transpose(0, 1)
        out[s:e] = F.scaled_dot_product_attention(qq, kk, vv, is_causal=True,
                                                  scale=scale).transpose(0, 1)
    return out.reshape(T, num_heads * head_dim).to(q.dtype)


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """``VocabParallelEmbedding.forward`` at tp=1 (layers/embed_head.py:43-52)."""
    return F.embedding(ids, table)


def last_token_l2(hidden: torch.Tensor, last_token_indices) -> torch.Tensor:
    """Post-process of ``GPUWorker._inference_worker`` (core/gpu_worker.py:253-261):
    gather the last token of each sequence, then ``F.normalize(p=2, dim=1)``
    (``x / max(||x||_2, 1e-12)``)."""
    idx = torch.as_tensor(last_token_indices, dtype=torch.int64)
    return F.normalize(hidden[idx].to(torch.float32), p=2, dim=1)
