"""AWQ int4 storage format and exact dequantisation, restated in numpy (oracle only).

The reference has no quantisation code: every linear layer is a dense ``F.linear``
(``layers/linear.py:54,86,179``).  AWQ is a new capability behind the same layer classes,
so its arithmetic is defined here and used as the bit-exact oracle for the CUDA
dequantisation.

Checkpoint format (AutoAWQ "GEMM" layout, the format vLLM's ``awq`` method loads):

* ``qweight`` int32 ``[K, N/8]``: word ``(k, j)`` holds the eight 4-bit codes
  ``q[k, 8j + AWQ_ORDER[i]]`` in bits ``[4i, 4i+4)``, ``AWQ_ORDER = [0,2,4,6,1,3,5,7]``.
  The order is pinned against vLLM 0.22.0
  ``vllm/model_executor/layers/quantization/utils/quant_utils.py`` ``awq_pack`` by the
  fixture ``tests/golden/awq_pack_vllm.npz``.
* ``qzeros`` int32 ``[K/G, N/8]``: zero-points packed the same way.
* ``scales`` fp16 ``[K/G, N]``.

Dequantisation (defined here; no reference pin exists): for group ``g = k // G``

    w[k, n] = (q[k, n] - z[g, n]) * s[g, n]

computed in fp32.  The product is exact in fp32 (|q - z| <= 15 has 4 significant bits
and an fp16 scale has 11).  The bf16 operand that the tensor cores consume is
``round_to_nearest_even_bf16(w)`` - exactly one rounding.

Kernel layout ("mes" layout, produced once at load time by ``mes_awq_repack``):

* ``qweight_mes`` int32 ``[K/8, N]``: word ``(b, n)`` holds ``q[8b + AWQ_ORDER[i], n]``
  in bits ``[4i, 4i+4)`` - the same interleave, applied along K instead of N, so that
  one word yields the bf16 pairs ``(k, k+1)`` of a single output column.
"""
from __future__ import annotations

import numpy as np

AWQ_ORDER = np.array([0, 2, 4, 6, 1, 3, 5, 7], dtype=np.int64)
PACK = 8


def _pack_last(q: np.ndarray) -> np.ndarray:
    """Pack uint8 codes ``[..., 8m]`` along the last axis into int32 ``[..., m]``."""
    q = np.asarray(q).astype(np.uint32)
    assert q.shape[-1] % PACK == 0
    g = q.reshape(*q.shape[:-1], q.shape[-1] // PACK, PACK)
    out = np.zeros(g.shape[:-1], dtype=np.uint32)
    for i in range(PACK):
        out |= (g[..., AWQ_ORDER[i]] & 0xF) << np.uint32(4 * i)
    return out.view(np.int32)


def _unpack_last(w: np.ndarray) -> np.ndarray:
    """Inverse of :func:`_pack_last`: int32 ``[..., m]`` -> uint8 ``[..., 8m]``."""
    w = np.ascontiguousarray(w).view(np.uint32)
    shifts = (4 * np.argsort(AWQ_ORDER)).astype(np.uint32)   # column c lives at nibble INV[c]
    out = ((w[..., None] >> shifts) & 0xF).astype(np.uint8)
    return out.reshape(*w.shape[:-1], w.shape[-1] * PACK)


def awq_pack(q: np.ndarray) -> np.ndarray:
    """uint8 codes ``[K, N]`` -> AWQ ``qweight``/``qzeros`` int32 ``[K, N/8]``."""
    return _pack_last(q)


def awq_unpack(qweight: np.ndarray) -> np.ndarray:
    """AWQ int32 ``[K, N/8]`` -> uint8 codes ``[K, N]``."""
    return _unpack_last(qweight)


def mes_repack(qweight: np.ndarray) -> np.ndarray:
    """AWQ ``qweight`` ``[K, N/8]`` -> kernel layout ``[K/8, N]`` (lossless)."""
    q = awq_unpack(qweight)                      # [K, N]
    return _pack_last(np.ascontiguousarray(q.T)).T.copy()  # pack along K -> [K/8, N]


def mes_unpack(qweight_mes: np.ndarray) -> np.ndarray:
    """Kernel layout ``[K/8, N]`` -> uint8 codes ``[K, N]``."""
    return np.ascontiguousarray(_unpack_last(np.ascontiguousarray(qweight_mes.T)).T)


def dequant_fp32(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray,
                 group_size: int = 128) -> np.ndarray:
    """Exact fp32 dequantisation ``(q - z) * s`` -> float32 ``[K, N]``."""
    q = awq_unpack(qweight).astype(np.int16)
    z = awq_unpack(qzeros).astype(np.int16)
    s = np.asarray(scales, dtype=np.float16).astype(np.float32)
    K, N = q.shape
    assert K % group_size == 0 and z.shape == (K // group_size, N) and s.shape == z.shape
    d = (q.reshape(K // group_size, group_size, N) - z[:, None, :]).astype(np.float32)
    return (d * s[:, None, :]).reshape(K, N)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round to nearest, ties to even); returns uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = (rounded & 0xFFFF).astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequant_bf16_bits(qweight, qzeros, scales, group_size: int = 128) -> np.ndarray:
    """The bf16 tensor-core operand: RNE_bf16((q - z) * s), as uint16 bits ``[K, N]``."""
    return f32_to_bf16_bits(dequant_fp32(qweight, qzeros, scales, group_size))


def random_awq(K: int, N: int, group_size: int = 128, seed: int = 0,
               scale_lo: float = 0.002, scale_hi: float = 0.02):
    """Seeded synthetic AWQ tensors with the distributions of the benchmark configs:
    codes and zero-points uniform in [0, 15], fp16 scales uniform in [scale_lo, scale_hi]."""
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, size=(K, N), dtype=np.uint8)
    z = rng.integers(0, 16, size=(K // group_size, N), dtype=np.uint8)
    s = rng.uniform(scale_lo, scale_hi, size=(K // group_size, N)).astype(np.float16)
    return awq_pack(q), awq_pack(z), s
