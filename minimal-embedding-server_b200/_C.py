"""ctypes binding of ``lib/libmes_b200.so`` (the C ABI declared in ``include/mes_b200.h``).

Every function here takes torch CUDA tensors, checks on the host that each tensor whose
pointer it passes lies on the same device and has the dtype, shape and layout the kernel
reads (a host pointer or a short buffer would otherwise reach the GPU), passes raw device
pointers plus the current CUDA stream to the library and raises :class:`MesError` on a
non-zero status.  There is no fallback: if the library is missing, fails to load, or no
CUDA device is present, the call raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libmes_b200.so")

_vp, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

# name -> (restype, argtypes); mirrors include/mes_b200.h
SIGNATURES = {
    "mes_version": (_i32, []),
    "mes_status_string": (ctypes.c_char_p, [_i32]),
    "mes_take_device_error": (_i32, [ctypes.POINTER(_i32)]),
    "mes_set_sm_reserve": (_i32, [_i32]),
    "mes_wait_probe": (_i32, [_i64, _i32, _vp]),
    "mes_embedding": (_i32, [_vp, _i64, _vp, _i64, _i64, _vp, _vp]),
    "mes_embedding_f32": (_i32, [_vp, _i64, _vp, _i64, _i64, _vp, _vp]),
    "mes_rmsnorm": (_i32, [_vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "mes_rmsnorm_f32in": (_i32, [_vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "mes_add_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "mes_add_rmsnorm_f32res": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "mes_qknorm_rope": (_i32, [_vp, _i64, _vp, _vp, _i32, _i64, _vp, _vp, _i64, _i32, _i32,
                               _i32, _f32, _i32, _vp]),
    "mes_silu_mul": (_i32, [_vp, _vp, _i64, _i64, _vp]),
    "mes_varlen_workspace_size": (_i64, [_i64]),
    "mes_varlen_schedule": (_i32, [_vp, _i64, _vp, _vp]),
    "mes_varlen_cu_seqlens": (_i32, [_vp, _i64, _vp, _vp, _vp]),
    "mes_varlen_attention": (_i32, [_vp, _i64, _vp, _vp, _i64, _i32, _i32, _i32, _f32, _vp]),
    "mes_varlen_attention_noalloc_max_tokens": (_i64, []),
    "mes_varlen_attention_noalloc": (_i32, [_vp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _f32,
                                            _vp]),
    "mes_last_token_l2": (_i32, [_vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "mes_awq_repack": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "mes_awq_dequant": (_i32, [_vp, _vp, _vp, _i64, _i64, _i32, _vp, _vp]),
    "mes_awq_gemm": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32,
                            _vp]),
    "mes_awq_gemm_residual": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                     _i32, _vp]),
    "mes_awq_gemm_silu": (_i32, [_vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32, _vp]),
    "mes_awq_gemm_workspace_size": (_i64, [_i64, _i64, _i64]),
    "mes_awq_panels": (_i32, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mes_awq_gemm_on_panel": (_i32, [_i32, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "mes_awq_gemm_ws": (_i32, [_i32, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                               _i32, _vp, _i64, _vp]),
}

_lib = None

# Number of kernel launches issued through this module (each wrapper below launches
# exactly one kernel); read by the benchmark to report its launch count.
launch_count = 0

# Optional per-launch timing hook for the AWQ GEMM: when set to a list, every awq_gemm /
# awq_gemm_residual call appends (start_event, end_event, flops, (kind, M, N, K)) recorded
# on the launching stream.
gemm_events = None
# Epilogue kinds ("bf16", "residual", "silu") whose GEMMs append to gemm_events; None = all.
gemm_event_kinds = None


def _timing_event():
    # external: inside a CUDA-graph capture the record becomes a graph node, so the events
    # time the kernel on every replay
    return torch.cuda.Event(enable_timing=True, external=True)


class MesError(RuntimeError):
    """A mes_b200 library call returned a non-zero status."""


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raises if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MesError(f"mes_b200 CUDA library not found at {LIB_PATH}; "
                           "build it with __graft_entry__.build()")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def status_string(code: int) -> str:
    return lib().mes_status_string(code).decode()


def _check(code: int, what: str, launches: int = 1) -> None:
    global launch_count
    if code != 0:
        raise MesError(f"{what}: {status_string(code)} (status {code})")
    launch_count += launches


def _p(t):
    return None if t is None else t.data_ptr()   # c_void_p arguments take plain ints


_raw_stream = torch._C._cuda_getCurrentRawStream


def _stream(t: torch.Tensor):
    if not t.is_cuda:
        raise MesError("mes_b200 kernels need CUDA tensors (there is no CPU path)")
    return _raw_stream(t.device.index)


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise MesError(msg)


def _arg(t, name: str, like: torch.Tensor, dtype=None, shape=None, contiguous: bool = False,
         unit_stride: bool = False) -> None:
    """Check the tensor argument ``t`` (None passes) before its pointer goes to a kernel: on
    ``like``'s device, of ``dtype`` (a dtype or a tuple of them), of ``shape``, contiguous
    or with unit inner stride when asked."""
    if t is None:
        return
    if t.device != like.device:
        raise MesError(f"{name} is on {t.device}, the kernel runs on {like.device}")
    if dtype is not None and t.dtype not in (dtype if isinstance(dtype, tuple) else (dtype,)):
        raise MesError(f"{name} must be {dtype}, got {t.dtype}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise MesError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if contiguous and not t.is_contiguous():
        raise MesError(f"{name} must be contiguous")
    if unit_stride and t.stride(-1) != 1:
        raise MesError(f"{name} must have unit inner stride")


_SCALES = (torch.int16, torch.float16)   # fp16 scales, or their int16 bit pattern


def _awq_args(qweight_mes, qzeros, scales, like: torch.Tensor, group_size: int) -> None:
    """Kernel-layout AWQ tensors: qweight_mes i32 [K/8, N], qzeros i32 [K/G, N/8], scales
    fp16 (or int16 bits) [K/G, N], all contiguous on ``like``'s device."""
    _need(qweight_mes.dim() == 2 and group_size > 0, "qweight_mes must be int32 [K/8, N]")
    K, N = qweight_mes.shape[0] * 8, qweight_mes.shape[1]
    _arg(qweight_mes, "qweight_mes", like, torch.int32, contiguous=True)
    _arg(qzeros, "qzeros", like, torch.int32, (K // group_size, N // 8), contiguous=True)
    _arg(scales, "scales", like, _SCALES, (K // group_size, N), contiguous=True)


def take_device_error() -> int:
    code = _i32(0)
    _check(lib().mes_take_device_error(ctypes.byref(code)), "mes_take_device_error", 0)
    return code.value


def set_sm_reserve(sms: int) -> None:
    """Keep ``sms`` SMs free of the persistent kernels (see ``mes_set_sm_reserve``)."""
    _check(lib().mes_set_sm_reserve(int(sms)), "mes_set_sm_reserve", 0)


# --------------------------------------------------------------------------------------
# torch-facing wrappers
# --------------------------------------------------------------------------------------
def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None):
    _need(ids.dtype == torch.int64 and ids.dim() == 1, "ids must be int64 [T]")
    _need(table.dtype == torch.bfloat16 and table.dim() == 2 and table.is_contiguous(),
          "table must be contiguous bf16 [vocab, H]")
    T, (V, H) = ids.shape[0], table.shape
    _arg(ids, "ids", table)
    _arg(out, "out", table, torch.bfloat16, (T, H), contiguous=True)
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=table.device)
    ids = ids.contiguous()
    _check(lib().mes_embedding(_p(ids), T, _p(table), V, H, _p(out), _stream(table)),
           "mes_embedding")
    return out


def embedding_f32(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None):
    """Gather widened to fp32 (the start of the fp32 residual stream)."""
    _need(ids.dtype == torch.int64 and ids.dim() == 1, "ids must be int64 [T]")
    _need(table.dtype == torch.bfloat16 and table.dim() == 2 and table.is_contiguous(),
          "table must be contiguous bf16 [vocab, H]")
    T, (V, H) = ids.shape[0], table.shape
    _arg(ids, "ids", table)
    _arg(out, "out", table, torch.float32, (T, H), contiguous=True)
    if out is None:
        out = torch.empty(T, H, dtype=torch.float32, device=table.device)
    _check(lib().mes_embedding_f32(_p(ids.contiguous()), T, _p(table), V, H, _p(out),
                                   _stream(table)), "mes_embedding_f32")
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None):
    """bf16 RMSNorm of a bf16 or fp32 ``x`` (fp32: the residual stream)."""
    _need(x.dtype in (torch.bfloat16, torch.float32) and x.is_contiguous(),
          "x must be contiguous bf16 or fp32")
    H = x.shape[-1]
    _need(x.dim() >= 1 and H > 0, "x must be [..., H] with H > 0")
    _arg(w, "w", x, torch.bfloat16, (H,), contiguous=True)
    _arg(out, "out", x, torch.bfloat16, x.shape, contiguous=True)
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    fn = lib().mes_rmsnorm if x.dtype == torch.bfloat16 else lib().mes_rmsnorm_f32in
    _check(fn(_p(x), _p(w), _p(out), x.numel() // H, H, eps, _stream(x)), "mes_rmsnorm")
    return out


def add_rmsnorm_f32res(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """residual (fp32, in place) += x (bf16); returns bf16 RMSNorm(residual)."""
    _need(x.dtype == torch.bfloat16 and residual.dtype == torch.float32, "bf16 x, fp32 residual")
    _need(x.is_contiguous() and residual.is_contiguous() and x.shape == residual.shape,
          "x and residual must be contiguous and of one shape")
    H = x.shape[-1]
    _need(x.dim() >= 1 and H > 0, "x must be [..., H] with H > 0")
    _arg(residual, "residual", x)
    _arg(w, "w", x, torch.bfloat16, (H,), contiguous=True)
    _arg(out, "out", x, torch.bfloat16, x.shape, contiguous=True)
    out = torch.empty_like(x) if out is None else out
    _check(lib().mes_add_rmsnorm_f32res(_p(x), _p(residual), _p(w), _p(out), x.numel() // H, H,
                                        eps, _stream(x)), "mes_add_rmsnorm_f32res")
    return out


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                out: torch.Tensor | None = None, residual_out: torch.Tensor | None = None):
    _need(x.dtype == torch.bfloat16 and residual.dtype == torch.bfloat16, "bf16 inputs")
    _need(x.is_contiguous() and residual.is_contiguous() and x.shape == residual.shape,
          "x and residual must be contiguous and of one shape")
    H = x.shape[-1]
    _need(x.dim() >= 1 and H > 0, "x must be [..., H] with H > 0")
    _arg(residual, "residual", x)
    _arg(w, "w", x, torch.bfloat16, (H,), contiguous=True)
    _arg(out, "out", x, torch.bfloat16, x.shape, contiguous=True)
    _arg(residual_out, "residual_out", x, torch.bfloat16, x.shape, contiguous=True)
    out = torch.empty_like(x) if out is None else out
    residual_out = torch.empty_like(residual) if residual_out is None else residual_out
    _check(lib().mes_add_rmsnorm(_p(x), _p(residual), _p(w), _p(out), _p(residual_out),
                                 x.numel() // H, H, eps, _stream(x)), "mes_add_rmsnorm")
    return out, residual_out


def qknorm_rope(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                num_q_heads: int, num_k_heads: int, head_dim: int,
                q_weight: torch.Tensor | None = None, k_weight: torch.Tensor | None = None,
                eps: float = 1e-6) -> torch.Tensor:
    """In place on ``qkv`` (rows of pitch ``qkv.stride(0)``): optional per-head RMSNorm of
    the first ``num_q_heads`` (weight ``q_weight``) and next ``num_k_heads`` heads
    (``k_weight``), then NeoX RoPE with ``cos_sin[positions]``."""
    _need(qkv.dtype == torch.bfloat16 and qkv.stride(-1) == 1, "qkv must be bf16, unit stride")
    _need(positions.dtype == torch.int64, "positions must be int64")
    _need(cos_sin.dtype in (torch.float32, torch.bfloat16) and cos_sin.is_contiguous(),
          "cos_sin must be a contiguous fp32/bf16 cache")
    apply_norm = q_weight is not None or k_weight is not None
    _need(positions.dim() == 1 and qkv.dim() == 2 and qkv.shape[0] == positions.shape[0],
          "qkv must be [T, ...] for positions [T]")
    _need(cos_sin.dim() == 2 and cos_sin.shape[1] == head_dim, "cos_sin must be [max_pos, D]")
    _arg(positions, "positions", qkv)
    _arg(cos_sin, "cos_sin", qkv)
    _arg(q_weight, "q_weight", qkv, torch.bfloat16, (head_dim,), contiguous=True)
    _arg(k_weight, "k_weight", qkv, torch.bfloat16, (head_dim,), contiguous=True)
    T = positions.shape[0]
    _check(lib().mes_qknorm_rope(_p(qkv), qkv.stride(0), _p(positions.contiguous()),
                                 _p(cos_sin), int(cos_sin.dtype == torch.float32),
                                 cos_sin.shape[0], _p(q_weight), _p(k_weight), T, num_q_heads,
                                 num_k_heads, head_dim, eps, int(apply_norm), _stream(qkv)),
           "mes_qknorm_rope")
    return qkv


def silu_mul(x: torch.Tensor, out: torch.Tensor | None = None):
    _need(x.dtype == torch.bfloat16 and x.is_contiguous() and x.shape[-1] % 2 == 0,
          "x must be contiguous bf16 [..., 2I]")
    I = x.shape[-1] // 2
    _arg(out, "out", x, torch.bfloat16, (*x.shape[:-1], I), contiguous=True)
    if out is None:
        out = torch.empty(*x.shape[:-1], I, dtype=x.dtype, device=x.device)
    _check(lib().mes_silu_mul(_p(x), _p(out), x.numel() // (2 * I), I, _stream(x)),
           "mes_silu_mul")
    return out


def varlen_workspace_size(T: int) -> int:
    return int(lib().mes_varlen_workspace_size(T))


def varlen_schedule(positions: torch.Tensor, workspace: torch.Tensor | None = None):
    _need(positions.dtype == torch.int64 and positions.dim() == 1, "positions must be int64 [T]")
    T = positions.shape[0]
    size = varlen_workspace_size(T)
    if workspace is None:
        workspace = torch.empty(size, dtype=torch.uint8, device=positions.device)
    _arg(workspace, "workspace", positions, torch.uint8, contiguous=True)
    _need(workspace.numel() >= size, "workspace too small")
    positions = positions.contiguous()
    _check(lib().mes_varlen_schedule(_p(positions), T, _p(workspace), _stream(positions)),
           "mes_varlen_schedule")
    return workspace


def varlen_cu_seqlens(workspace: torch.Tensor, T: int):
    _need(workspace.dtype == torch.uint8 and workspace.numel() >= varlen_workspace_size(T),
          "workspace must be the uint8 schedule of a batch of T tokens")
    cu = torch.empty(T + 1, dtype=torch.int32, device=workspace.device)
    n = torch.empty(1, dtype=torch.int32, device=workspace.device)
    _check(lib().mes_varlen_cu_seqlens(_p(workspace), T, _p(cu), _p(n), _stream(workspace)),
           "mes_varlen_cu_seqlens", 0)
    return cu, n


def varlen_attention(qkv: torch.Tensor, workspace: torch.Tensor, num_heads: int,
                     num_kv_heads: int, head_dim: int, scale: float,
                     out: torch.Tensor | None = None):
    _need(qkv.dtype == torch.bfloat16 and qkv.dim() == 2 and qkv.stride(-1) == 1,
          "qkv must be bf16 [T, (Hq + 2 Hkv) D], unit stride")
    T = qkv.shape[0]
    _arg(workspace, "workspace", qkv, torch.uint8, contiguous=True)
    _need(workspace.numel() >= varlen_workspace_size(T), "workspace too small for T tokens")
    _arg(out, "out", qkv, torch.bfloat16, (T, num_heads * head_dim), contiguous=True)
    if out is None:
        out = torch.empty(T, num_heads * head_dim, dtype=torch.bfloat16, device=qkv.device)
    _check(lib().mes_varlen_attention(_p(qkv), qkv.stride(0), _p(out), _p(workspace), T,
                                      num_heads, num_kv_heads, head_dim, scale, _stream(qkv)),
           "mes_varlen_attention")
    return out


def last_token_l2(hidden: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None):
    _need(hidden.dtype == torch.bfloat16 and hidden.is_contiguous() and hidden.dim() == 2,
          "hidden must be contiguous bf16 [T, H]")
    _need(idx.dtype == torch.int64 and idx.dim() == 1, "indices must be int64 [B]")
    T, H = hidden.shape
    B = idx.shape[0]
    _arg(idx, "indices", hidden)
    _arg(out, "out", hidden, torch.float32, (B, H), contiguous=True)
    if out is None:
        out = torch.empty(B, H, dtype=torch.float32, device=hidden.device)
    _check(lib().mes_last_token_l2(_p(hidden), T, H, _p(idx.contiguous()), B, _p(out),
                                   _stream(hidden)), "mes_last_token_l2")
    return out


def awq_repack(qweight: torch.Tensor) -> torch.Tensor:
    _need(qweight.dtype == torch.int32 and qweight.dim() == 2 and qweight.is_contiguous(),
          "qweight must be contiguous int32 [K, N/8]")
    K, N = qweight.shape[0], qweight.shape[1] * 8
    out = torch.empty(K // 8, N, dtype=torch.int32, device=qweight.device)
    _check(lib().mes_awq_repack(_p(qweight), K, N, _p(out), _stream(qweight)), "mes_awq_repack")
    return out


def awq_dequant(qweight_mes: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                group_size: int = 128) -> torch.Tensor:
    """bf16 W^T [N, K] with the GEMM's exact dequantisation (for verification)."""
    _awq_args(qweight_mes, qzeros, scales, qweight_mes, group_size)
    K, N = qweight_mes.shape[0] * 8, qweight_mes.shape[1]
    out = torch.empty(N, K, dtype=torch.bfloat16, device=qweight_mes.device)
    _check(lib().mes_awq_dequant(_p(qweight_mes), _p(qzeros), _p(scales), K, N, group_size,
                                 _p(out), _stream(qweight_mes)), "mes_awq_dequant")
    return out


# Epilogue selectors of mes_awq_gemm_ws.
EPI_BF16, EPI_RESIDUAL, EPI_SILU = 0, 1, 2
_EPI_NAME = {EPI_BF16: "bf16", EPI_RESIDUAL: "residual", EPI_SILU: "silu"}

# Whether the GEMM wrappers hand the library a weight-panel workspace (taken from the torch
# caching allocator, or from a CUDA graph's pool during capture).  Without one the library
# runs its fused dequantising kernels for every M.
use_gemm_workspace = True


def gemm_uses_panel(M: int, N: int, K: int) -> bool:
    """Whether a GEMM of this shape runs on a dequantised weight panel (M > 1024 tokens,
    N % 256 == 0), when the wrappers use workspaces at all."""
    return use_gemm_workspace and int(lib().mes_awq_gemm_workspace_size(M, N, K)) > 0


def awq_panels(weights, panels) -> None:
    """Build the bf16 weight panels ``panels[i]`` (``[N, K]``, from ``torch.empty``) of the
    kernel-layout AWQ tensors ``weights[i] = (qweight_mes, qzeros, scales)`` in one launch
    (``mes_awq_panels``; at most 8)."""
    n = len(weights)
    _need(0 < n <= 8 and len(panels) == n, "1..8 panels")
    arr = lambda vals, t: (t * n)(*vals)
    qw = arr([_p(w[0]) for w in weights], _vp)
    qz = arr([_p(w[1]) for w in weights], _vp)
    sc = arr([_p(w[2]) for w in weights], _vp)
    K = arr([w[0].shape[0] * 8 for w in weights], _i64)
    N = arr([w[0].shape[1] for w in weights], _i64)
    for (w, p_) in zip(weights, panels):
        _awq_args(*w, panels[0], 128)
        _arg(p_, "panel", panels[0], torch.bfloat16, (w[0].shape[1], w[0].shape[0] * 8),
             contiguous=True)
    _check(lib().mes_awq_panels(n, qw, qz, sc, K, N, arr([_p(p_) for p_ in panels], _vp),
                                _stream(panels[0])), "mes_awq_panels")


def _awq_gemm_call(epi: int, x: torch.Tensor, qweight_mes: torch.Tensor, qzeros: torch.Tensor,
                   scales: torch.Tensor, bias, y: torch.Tensor, group_size: int,
                   panel: torch.Tensor | None = None) -> None:
    _awq_args(qweight_mes, qzeros, scales, x, group_size)
    K, N = qweight_mes.shape[0] * 8, qweight_mes.shape[1]
    M = x.shape[0]
    _arg(bias, "bias", x, torch.bfloat16, (N,), contiguous=True)
    _arg(y, "output", x, unit_stride=True)
    _arg(panel, "panel", x)
    ev = gemm_events if gemm_event_kinds is None or _EPI_NAME[epi] in gemm_event_kinds else None
    if ev is not None:
        e0, e1 = _timing_event(), _timing_event()
        e0.record()
    if panel is not None and gemm_uses_panel(M, N, K):
        _need(tuple(panel.shape) == (N, K) and panel.dtype == torch.bfloat16, "panel must be bf16 [N, K]")
        _check(lib().mes_awq_gemm_on_panel(epi, _p(x), x.stride(0), _p(panel), _p(bias), _p(y),
                                           y.stride(0), M, N, K, _stream(x)),
               f"mes_awq_gemm_on_panel ({_EPI_NAME[epi]} epilogue)")
    else:
        ws_bytes = int(lib().mes_awq_gemm_workspace_size(M, N, K)) if use_gemm_workspace else 0
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes > 0 else None
        _check(lib().mes_awq_gemm_ws(epi, _p(x), x.stride(0), _p(qweight_mes), _p(qzeros),
                                     _p(scales), _p(bias), _p(y), y.stride(0), M, N, K, group_size,
                                     _p(ws), ws_bytes, _stream(x)),
               f"mes_awq_gemm ({_EPI_NAME[epi]} epilogue)", 2 if ws is not None else 1)
    if ev is not None:
        e1.record()
        ev.append((e0, e1, 2.0 * M * N * K, (_EPI_NAME[epi], M, N, K)))


def awq_gemm_residual(x: torch.Tensor, qweight_mes: torch.Tensor, qzeros: torch.Tensor,
                      scales: torch.Tensor, residual: torch.Tensor,
                      bias: torch.Tensor | None = None, group_size: int = 128,
                      panel: torch.Tensor | None = None) -> torch.Tensor:
    """``residual[M, N] (fp32) += x @ W (+ bias)`` in the GEMM epilogue."""
    _need(x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(-1) == 1,
          "x must be bf16 [M, K] with unit inner stride")
    _need(residual.dtype == torch.float32 and residual.stride(-1) == 1, "fp32 residual")
    K, N = qweight_mes.shape[0] * 8, qweight_mes.shape[1]
    M = x.shape[0]
    _need(x.shape[1] == K and residual.dim() == 2 and tuple(residual.shape) == (M, N),
          "shape mismatch")
    _awq_gemm_call(EPI_RESIDUAL, x, qweight_mes, qzeros, scales, bias, residual, group_size, panel)
    return residual


def awq_gemm_silu(x: torch.Tensor, qweight_mes: torch.Tensor, qzeros: torch.Tensor,
                  scales: torch.Tensor, out: torch.Tensor | None = None,
                  group_size: int = 128, panel: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(x @ Wg) * (x @ Wu)`` with the gate/up columns interleaved in blocks of 16
    (see ``interleave_gate_up``); output ``[M, N/2]`` bf16."""
    _need(x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(-1) == 1,
          "x must be bf16 [M, K] with unit inner stride")
    K, N = qweight_mes.shape[0] * 8, qweight_mes.shape[1]
    M = x.shape[0]
    _need(x.shape[1] == K, f"x has K={x.shape[1]}, weight has K={K}")
    _arg(out, "out", x, torch.bfloat16, (M, N // 2), unit_stride=True)
    if out is None:
        out = torch.empty(M, N // 2, dtype=torch.bfloat16, device=x.device)
    _awq_gemm_call(EPI_SILU, x, qweight_mes, qzeros, scales, None, out, group_size, panel)
    return out


def interleave_gate_up(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor):
    """Permute AWQ tensors of a ``[gate | up]`` projection (N = 2I columns) so that blocks of
    16 gate and 16 up columns alternate, the layout ``mes_awq_gemm_silu`` expects."""
    N = scales.shape[1]
    I = N // 2
    _need(I % 16 == 0, "the intermediate size per rank must be a multiple of 16")
    blocks = torch.arange(I // 16, device=scales.device)
    cols = torch.stack([blocks * 16, I + blocks * 16], dim=1).reshape(-1)        # block starts
    perm = (cols[:, None] + torch.arange(16, device=scales.device)).reshape(-1)  # [N]
    perm8 = perm[::8] // 8                                                       # packed columns
    return (qweight.index_select(1, perm8).contiguous(), qzeros.index_select(1, perm8).contiguous(),
            scales.index_select(1, perm).contiguous())


def awq_gemm(x: torch.Tensor, qweight_mes: torch.Tensor, qzeros: torch.Tensor,
             scales: torch.Tensor, bias: torch.Tensor | None = None,
             out: torch.Tensor | None = None, group_size: int = 128,
             panel: torch.Tensor | None = None) -> torch.Tensor:
    """``x[M, K] @ W[K, N] (+ bias)`` with W given by AWQ tensors in the kernel layout."""
    _need(x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(-1) == 1,
          "x must be bf16 [M, K] with unit inner stride")
    K, N = qweight_mes.shape[0] * 8, qweight_mes.shape[1]
    M = x.shape[0]
    _need(x.shape[1] == K, f"x has K={x.shape[1]}, weight has K={K}")
    _arg(out, "out", x, torch.bfloat16, (M, N), unit_stride=True)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    _awq_gemm_call(EPI_BF16, x, qweight_mes, qzeros, scales, bias, out, group_size, panel)
    return out
