"""Tensor-parallel linear layers with AWQ int4 weights.

Same classes, constructor arguments and ``weight_loader`` conventions as the reference's
``layers/linear.py`` (``ReplicatedLinear:31``, ``ColumnParallelLinear:57``,
``MergedColumnParallelLinear:90``, ``QKVParallelLinear:110``, ``RowParallelLinear:147``);
TP rank and size come from ``torch.distributed`` at construction (``linear.py:24-25``).
The reference stores a dense ``weight [out, in]`` and calls ``F.linear``; here each layer
stores the AWQ checkpoint tensors of its shard

* ``qweight`` int32 ``[K, N/8]``, ``qzeros`` int32 ``[K/G, N/8]``,
* ``scales`` fp16 ``[K/G, N]`` - held as its int16 bit pattern so that ``model.to(dtype)``
  (``core/gpu_worker.py:89-93``) cannot re-round it,
* ``bias`` bf16 ``[N]`` when requested,

and computes ``x @ W (+ bias)`` with the tcgen05 W4A16 kernel (``mes_awq_gemm``).  The
output dimension of a column-parallel layer is sharded on the packed axis (``N/8``), the
input dimension of a row-parallel layer on ``K`` and on ``K/G`` for zeros/scales, so every
shard keeps whole quantisation groups.  ``RowParallelLinear`` adds its bias on rank 0 only
and sums the partial outputs with an NCCL all-reduce (``linear.py:176-180``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from .. import _C

GROUP_SIZE = 128
PACK = 8


def divide(numerator: int, denominator: int) -> int:
    """``linear.py:7-9``."""
    assert numerator % denominator == 0, f"{numerator} is not divisible by {denominator}"
    return numerator // denominator


def _tp():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


class AWQConfig:
    """Quantisation parameters of the AWQ checkpoints this package loads."""

    def __init__(self, group_size: int = GROUP_SIZE, bits: int = 4):
        if bits != 4 or group_size != GROUP_SIZE:
            raise ValueError("only 4-bit AWQ with group_size 128 is supported")
        self.group_size = group_size
        self.bits = bits


class LinearBase(nn.Module):
    """``linear.py:12-28`` with AWQ parameters for a local ``[in_local, out_local]`` shard."""

    def __init__(self, input_size: int, output_size: int, tp_dim: int | None = None,
                 quant_config: AWQConfig | None = None):
        super().__init__()
        self.input_size = input_size
        self.output_size = output_size
        self.tp_dim = tp_dim
        self.tp_rank, self.tp_size = _tp()
        self.quant_config = quant_config or AWQConfig()
        self.group_size = self.quant_config.group_size
        self._qweight_mes = None  # kernel layout, built by process_weights_after_loading()
        # bf16 weight panel W^T [n_local, k_local] prepared by the owning decoder layer for
        # the current forward (see DecoderLayer.build_panels); None: the GEMM builds its own.
        self.panel = None

    def _create_weights(self, k_local: int, n_local: int, bias: bool, bias_size: int):
        G = self.group_size
        if k_local % G or n_local % PACK:
            raise ValueError(f"AWQ shard [{k_local}, {n_local}] must have K % {G} == 0 "
                             f"and N % {PACK} == 0")
        self.k_local, self.n_local = k_local, n_local
        self.qweight = nn.Parameter(torch.zeros(k_local, n_local // PACK, dtype=torch.int32),
                                    requires_grad=False)
        self.qzeros = nn.Parameter(torch.zeros(k_local // G, n_local // PACK, dtype=torch.int32),
                                   requires_grad=False)
        self.scales = nn.Parameter(torch.zeros(k_local // G, n_local, dtype=torch.int16),
                                   requires_grad=False)
        for p in (self.qweight, self.qzeros, self.scales):
            p.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.zeros(bias_size, dtype=torch.bfloat16),
                                     requires_grad=False)
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    # ------------------------------------------------------------------ loading helpers
    @staticmethod
    def _as_stored(param: nn.Parameter, loaded: torch.Tensor) -> torch.Tensor:
        """Checkpoint tensor -> the dtype the parameter stores (fp16 scales as int16 bits)."""
        if param.dtype == torch.int16:
            return loaded.to(torch.float16).view(torch.int16)
        return loaded.to(param.dtype)

    def _param_kind(self, param) -> str:
        for name in ("qweight", "qzeros", "scales", "bias"):
            if getattr(self, name, None) is param:
                return name
        raise ValueError("unknown parameter")

    def _out_slice(self, kind: str, start: int, size: int) -> tuple[int, int]:
        if kind in ("qweight", "qzeros"):
            assert start % PACK == 0 and size % PACK == 0, "column shards must be multiples of 8"
            return start // PACK, size // PACK
        return start, size

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, *args):
        param.data.copy_(self._as_stored(param, loaded_weight))
        self._qweight_mes = None

    # ------------------------------------------------------------------ compute
    def process_weights_after_loading(self):
        """Repack ``qweight`` into the kernel layout on the parameter's device (once)."""
        self._qweight_mes = _C.awq_repack(self.qweight.data.contiguous())

    def gemm_weights(self):
        """``(qweight_mes, qzeros, scales)`` of the kernel layout this layer's GEMM uses."""
        if self._qweight_mes is None or self._qweight_mes.device != self.qweight.device:
            self.process_weights_after_loading()
        return self._qweight_mes, self.qzeros, self.scales

    def _mm(self, x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
        """Plain GEMM in the checkpoint's column order (the prepared panel is used only when
        it was built from these weights, not from a fused-epilogue layout)."""
        qw, qz, sc = LinearBase.gemm_weights(self)
        panel = self.panel if self.gemm_weights()[0] is qw else None
        shape = x.shape
        y = _C.awq_gemm(x.reshape(-1, shape[-1]), qw, qz, sc, bias, group_size=self.group_size,
                        panel=panel)
        return y.view(*shape[:-1], y.shape[-1])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class ReplicatedLinear(LinearBase):
    """``linear.py:31-54``: the full weight on every rank."""

    def __init__(self, input_size: int, output_size: int, bias: bool = False,
                 quant_config: AWQConfig | None = None):
        super().__init__(input_size, output_size, None, quant_config)
        self._create_weights(input_size, output_size, bias, output_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._mm(x, self.bias)


class ColumnParallelLinear(LinearBase):
    """``linear.py:57-83``: output features sharded across ranks."""

    def __init__(self, input_size: int, output_size: int, bias: bool = False,
                 quant_config: AWQConfig | None = None):
        super().__init__(input_size, output_size, 0, quant_config)
        self.input_size_per_partition = input_size
        self.output_size_per_partition = divide(output_size, self.tp_size)
        self._create_weights(input_size, self.output_size_per_partition, bias,
                             self.output_size_per_partition)

    def _load_out_range(self, param, loaded: torch.Tensor, dst_start: int, dst_size: int,
                        src_start: int):
        """Copy output features [src_start, src_start+dst_size) of a full checkpoint tensor
        into features [dst_start, dst_start+dst_size) of this shard."""
        kind = self._param_kind(param)
        axis = 0 if kind == "bias" else 1
        d0, dn = self._out_slice(kind, dst_start, dst_size)
        s0, sn = self._out_slice(kind, src_start, dst_size)
        param.data.narrow(axis, d0, dn).copy_(
            self._as_stored(param, loaded.narrow(axis, s0, sn)))
        self._qweight_mes = None

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, *args):
        n = self.output_size_per_partition
        self._load_out_range(param, loaded_weight, 0, n, self.tp_rank * n)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._mm(x, self.bias)


class MergedColumnParallelLinear(ColumnParallelLinear):
    """``linear.py:90-107``: ``[gate | up]`` per rank; shard ``i`` of every checkpoint
    tensor is chunked across ranks and placed at ``sum(output_sizes[:i]) / tp``."""

    def __init__(self, input_size: int, output_sizes: list[int], bias: bool = False,
                 quant_config: AWQConfig | None = None):
        self.output_sizes = list(output_sizes)
        super().__init__(input_size, sum(output_sizes), bias=bias, quant_config=quant_config)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor,
                      loaded_shard_id: int):
        tp = self.tp_size
        offset = sum(self.output_sizes[:loaded_shard_id]) // tp
        size = self.output_sizes[loaded_shard_id] // tp
        self._load_out_range(param, loaded_weight, offset, size, self.tp_rank * size)
        self._silu_pack = None

    def process_weights_after_loading(self):
        """Build the kernel layout the model will use: the gate/up-interleaved pack for the
        fused SiLU GEMM when it applies (the plain layout is then built only on demand)."""
        if self.supports_silu():
            self._silu_pack = None
            self._silu_pack = self._build_silu_pack()
        else:
            super().process_weights_after_loading()

    def _build_silu_pack(self):
        qw, qz, sc = _C.interleave_gate_up(self.qweight.data, self.qzeros.data, self.scales.data)
        return (_C.awq_repack(qw), qz, sc)

    def supports_silu(self) -> bool:
        """Whether forward_silu applies: two equal halves, 64-aligned per rank, no bias."""
        return (len(self.output_sizes) == 2 and self.output_sizes[0] == self.output_sizes[1]
                and (self.output_size_per_partition // 2) % 64 == 0
                and self.output_size_per_partition % 128 == 0 and self.bias is None)

    def gemm_weights(self):
        """The gate/up-interleaved pack when the fused SiLU GEMM applies, else the plain
        kernel layout."""
        if not self.supports_silu():
            return super().gemm_weights()
        pack = getattr(self, "_silu_pack", None)
        if pack is None or pack[0].device != self.qweight.device:
            pack = self._silu_pack = self._build_silu_pack()
        return pack

    def forward_silu(self, x: torch.Tensor) -> torch.Tensor:
        """``SiluAndMul(self(x))`` as one GEMM: the epilogue multiplies silu(gate) by up
        (``layers/activation.py:12-14``), so the [T, 2I] projection never reaches HBM."""
        pack = self.gemm_weights()
        shape = x.shape
        y = _C.awq_gemm_silu(x.reshape(-1, shape[-1]), *pack, group_size=self.group_size,
                             panel=self.panel)
        return y.view(*shape[:-1], y.shape[-1])


class QKVParallelLinear(ColumnParallelLinear):
    """``linear.py:110-144``: local output ``[q | k | v]`` with ``num_heads`` and
    ``num_kv_heads`` heads of ``head_size`` per rank."""

    def __init__(self, hidden_size: int, head_size: int, total_num_heads: int,
                 total_num_kv_heads: int | None = None, bias: bool = False,
                 quant_config: AWQConfig | None = None):
        self.head_size = head_size
        self.total_num_heads = total_num_heads
        self.total_num_kv_heads = total_num_kv_heads or total_num_heads
        _, tp_size = _tp()
        self.num_heads = divide(self.total_num_heads, tp_size)
        self.num_kv_heads = divide(self.total_num_kv_heads, tp_size)
        output_size = (self.total_num_heads + 2 * self.total_num_kv_heads) * head_size
        super().__init__(hidden_size, output_size, bias, quant_config)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor,
                      loaded_shard_id: str):
        assert loaded_shard_id in ("q", "k", "v")
        D = self.head_size
        if loaded_shard_id == "q":
            size, offset = self.num_heads * D, 0
        elif loaded_shard_id == "k":
            size, offset = self.num_kv_heads * D, self.num_heads * D
        else:
            size, offset = self.num_kv_heads * D, (self.num_heads + self.num_kv_heads) * D
        self._load_out_range(param, loaded_weight, offset, size, self.tp_rank * size)


class RowParallelLinear(LinearBase):
    """``linear.py:147-180``: input features sharded; partial outputs all-reduced."""

    def __init__(self, input_size: int, output_size: int, bias: bool = False,
                 quant_config: AWQConfig | None = None):
        super().__init__(input_size, output_size, 1, quant_config)
        self.input_size_per_partition = divide(input_size, self.tp_size)
        self.output_size_per_partition = output_size
        self._create_weights(self.input_size_per_partition, output_size, bias, output_size)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor, *args):
        kind = self._param_kind(param)
        if kind == "bias":
            param.data.copy_(self._as_stored(param, loaded_weight))
        else:
            rows = param.data.shape[0]
            param.data.copy_(self._as_stored(
                param, loaded_weight.narrow(0, self.tp_rank * rows, rows)))
        self._qweight_mes = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self._mm(x, self.bias if self.tp_rank == 0 else None)
        if self.tp_size > 1:
            dist.all_reduce(y)
        return y

    def forward_partial(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's partial product (bias on rank 0), before the all-reduce - for callers
        that overlap the reduction with other work."""
        return self._mm(x, self.bias if self.tp_rank == 0 else None)

    def forward_residual(self, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor | None:
        """Add this projection to the fp32 residual stream.  At tp == 1 the add happens in
        the GEMM epilogue (returns None); at tp > 1 the bf16 partial products are summed
        with an all-reduce and returned for the following add+RMSNorm to apply."""
        if self.tp_size > 1:
            return self.forward(x)
        qw, qz, sc = self.gemm_weights()
        _C.awq_gemm_residual(x.reshape(-1, x.shape[-1]), qw, qz, sc,
                             residual.view(-1, residual.shape[-1]), self.bias,
                             group_size=self.group_size, panel=self.panel)
        return None
