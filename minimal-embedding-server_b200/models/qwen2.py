"""Qwen2 decoder (``models/qwen2.py``) on sm_100a kernels with AWQ int4 linears.

Module tree, parameter names and ``packed_modules_mapping`` match the reference so that
its checkpoint loader conventions apply.  As in the reference, attention has a QKV bias
and no q/k norm in ``forward`` (``qwen2.py:81-86``; the norm modules exist, unused), and
``Qwen2MLP`` (gate_up -> SiLU-and-mul -> down, ``:89-117``) is shared with Qwen3.

Residual stream.  The reference keeps the residual in bf16 and rounds every o_proj /
down_proj output to bf16 before adding it (``layernorm.py:30-41``).  Here the residual is
fp32 and the projection is accumulated into it inside the GEMM epilogue (tp == 1) or
after the all-reduce (tp > 1); the block's math is otherwise unchanged.  This removes two
bf16 roundings per block, which is what keeps full-depth embeddings within the 0.9995
cosine bound of the fp32 reference.  ``DecoderLayer.forward`` therefore passes
``(pending_delta, residual_fp32)`` between layers, where ``pending_delta`` is None when
the projection was already added.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import nn

from .. import _C
from ..layers.activation import SiluAndMul
from ..layers.attention import batch_schedule, create_attention
from ..layers.embed_head import VocabParallelEmbedding
from ..layers.layernorm import RMSNorm
from ..layers.linear import MergedColumnParallelLinear, QKVParallelLinear, RowParallelLinear
from ..layers.rotary_embedding import get_rope
from ..schemas.config import MESConfig
from .registry import register_model


def _tp_size() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def _rope_theta(cfg) -> float:
    theta = getattr(cfg, "rope_theta", None)
    if theta is None:
        params = getattr(cfg, "rope_parameters", None) or {}
        theta = params.get("rope_theta") if isinstance(params, dict) else None
    # The reference falls back to 1e6 when the config has no rope_theta (qwen3.py:113).
    return float(theta) if theta is not None else 1000000.0


class Qwen2Attention(nn.Module):

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int,
                 mes_config: MESConfig, max_position: int = 4096 * 32,
                 head_dim: int | None = None, rms_norm_eps: float = 1e-06,
                 qkv_bias: bool = False, rope_theta: float = 10000,
                 rope_scaling: tuple | None = None, qk_norm: bool = False) -> None:
        super().__init__()
        tp_size = _tp_size()
        self.total_num_heads = num_heads
        assert self.total_num_heads % tp_size == 0
        self.num_heads = self.total_num_heads // tp_size
        self.total_num_kv_heads = num_kv_heads
        assert self.total_num_kv_heads % tp_size == 0
        self.num_kv_heads = self.total_num_kv_heads // tp_size
        self.head_dim = head_dim or hidden_size // self.total_num_heads
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.scaling = self.head_dim ** -0.5
        self.mes_config = mes_config
        self.apply_qk_norm = qk_norm
        quant = mes_config.quant_config
        self.qkv_proj = QKVParallelLinear(hidden_size, self.head_dim, self.total_num_heads,
                                          self.total_num_kv_heads, bias=qkv_bias,
                                          quant_config=quant)
        self.o_proj = RowParallelLinear(self.total_num_heads * self.head_dim, hidden_size,
                                        bias=False, quant_config=quant)
        self.rotary_emb = get_rope(self.head_dim, rotary_dim=self.head_dim,
                                   max_position=max_position, base=rope_theta,
                                   rope_scaling=rope_scaling)
        self.attn = create_attention(self.num_heads, self.head_dim, self.scaling,
                                     self.num_kv_heads, attn_backend=mes_config.attn_backend)
        self.q_norm = RMSNorm(self.head_dim, eps=rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, eps=rms_norm_eps)

    def _attend(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
        qkv = self.qkv_proj(hidden_states)
        if self.apply_qk_norm:
            self.rotary_emb.forward_fused(positions, qkv, self.num_heads, self.num_kv_heads,
                                          self.q_norm, self.k_norm)
        else:
            self.rotary_emb.forward_fused(positions, qkv, self.num_heads, self.num_kv_heads)
        return self.attn.forward_packed(qkv, positions)

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
        """``qwen2.py:76-86`` / ``qwen3.py:76-92``: attention block output (bf16)."""
        return self.o_proj(self._attend(positions, hidden_states))

    def forward_residual(self, positions, hidden_states, residual):
        """Attention block added into the fp32 residual stream (see module docstring)."""
        return self.o_proj.forward_residual(self._attend(positions, hidden_states), residual)

    def forward_partial(self, positions, hidden_states):
        """This rank's o_proj partial product, before the all-reduce."""
        return self.o_proj.forward_partial(self._attend(positions, hidden_states))


class Qwen2MLP(nn.Module):

    def __init__(self, hidden_size: int, intermediate_size: int, hidden_act: str,
                 mes_config: MESConfig) -> None:
        super().__init__()
        self.mes_config = mes_config
        quant = mes_config.quant_config
        self.gate_up_proj = MergedColumnParallelLinear(hidden_size, [intermediate_size] * 2,
                                                       bias=False, quant_config=quant)
        self.down_proj = RowParallelLinear(intermediate_size, hidden_size, bias=False,
                                           quant_config=quant)
        assert hidden_act == "silu"
        self.act_fn = SiluAndMul()

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_up_proj(x)))

    def _act(self, x):
        if self.gate_up_proj.supports_silu():
            return self.gate_up_proj.forward_silu(x)   # GEMM with SiLU-and-mul epilogue
        return self.act_fn(self.gate_up_proj(x))

    def forward_residual(self, x, residual):
        return self.down_proj.forward_residual(self._act(x), residual)

    def forward_partial(self, x):
        """This rank's down_proj partial product, before the all-reduce."""
        return self.down_proj.forward_partial(self._act(x))


def _attn_kwargs(model_config, qkv_bias: bool, qk_norm: bool) -> dict:
    return dict(
        hidden_size=model_config.hidden_size,
        num_heads=model_config.num_attention_heads,
        num_kv_heads=model_config.num_key_value_heads,
        max_position=model_config.max_position_embeddings,
        rms_norm_eps=model_config.rms_norm_eps,
        qkv_bias=qkv_bias,
        head_dim=getattr(model_config, "head_dim", None),
        rope_theta=_rope_theta(model_config),
        rope_scaling=None,
        qk_norm=qk_norm,
    )


class DecoderLayer(nn.Module):
    """Pre-norm decoder block shared by Qwen2 and Qwen3 (``qwen2.py:120-165``,
    ``qwen3.py:94-139``)."""

    def __init__(self, mes_config: MESConfig, qkv_bias: bool, qk_norm: bool) -> None:
        super().__init__()
        self.mes_config = mes_config
        mc = mes_config.model_config
        self.self_attn = Qwen2Attention(mes_config=mes_config, **_attn_kwargs(mc, qkv_bias, qk_norm))
        self.mlp = Qwen2MLP(hidden_size=mc.hidden_size, intermediate_size=mc.intermediate_size,
                            hidden_act=mc.hidden_act, mes_config=mes_config)
        self.input_layernorm = RMSNorm(mc.hidden_size, eps=mc.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(mc.hidden_size, eps=mc.rms_norm_eps)

    def linears(self):
        return (self.self_attn.qkv_proj, self.self_attn.o_proj, self.mlp.gate_up_proj,
                self.mlp.down_proj)

    def build_panels(self, tokens: int) -> None:
        """Dequantise, in one launch, the weight panels of this block's projections whose
        GEMMs over ``tokens`` rows run on a panel (``mes_awq_panels``), and hand them to the
        layers for this forward.  Both micro-batches of the tensor-parallel overlap share
        them: a panel depends on the weights only."""
        use = [lin for lin in self.linears()
               if _C.gemm_uses_panel(tokens, lin.n_local, lin.k_local)]
        if not use:
            return
        sizes = [lin.n_local * lin.k_local for lin in use]
        buf = torch.empty(sum(sizes), dtype=torch.bfloat16, device=use[0].qweight.device)
        panels, off = [], 0
        for lin, n in zip(use, sizes):
            panels.append(buf[off:off + n].view(lin.n_local, lin.k_local))
            off += n
        _C.awq_panels([lin.gemm_weights() for lin in use], panels)
        for lin, p in zip(use, panels):
            lin.panel = p

    def clear_panels(self) -> None:
        for lin in self.linears():
            lin.panel = None

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor | None,
                residual: torch.Tensor | None):
        """One block on the fp32 residual stream.  First layer: ``hidden_states`` is the
        fp32 embedding, which becomes the residual.  Later layers: ``hidden_states`` is the
        previous block's pending delta (None once it was added in a GEMM epilogue)."""
        self.build_panels(positions.shape[0])
        try:
            if residual is None:
                residual = hidden_states
                x = self.input_layernorm.residual_norm(residual)
            else:
                x = self.input_layernorm.residual_norm(residual, hidden_states)
            delta = self.self_attn.forward_residual(positions, x, residual)
            x = self.post_attention_layernorm.residual_norm(residual, delta)
            delta = self.mlp.forward_residual(x, residual)
            return delta, residual
        finally:
            self.clear_panels()

    def forward_last_rows(self, positions: torch.Tensor, hidden_states: torch.Tensor | None,
                          residual: torch.Tensor | None, rows: torch.Tensor):
        """The block for the token rows ``rows`` (int64 [B]) only: attention still reads every
        token's keys and values, but o_proj, the MLP and the residual updates run on the B
        gathered rows.  Returns ``(pending_delta, residual_rows)`` like :meth:`forward`, for
        the B rows."""
        if residual is None:
            residual = hidden_states
            x = self.input_layernorm.residual_norm(residual)
        else:
            x = self.input_layernorm.residual_norm(residual, hidden_states)
        attn = self.self_attn._attend(positions, x).index_select(0, rows)
        res = residual.index_select(0, rows)
        delta = self.self_attn.o_proj.forward_residual(attn, res)
        x = self.post_attention_layernorm.residual_norm(res, delta)
        delta = self.mlp.forward_residual(x, res)
        return delta, res


class Qwen2DecoderLayer(DecoderLayer):

    def __init__(self, mes_config: MESConfig) -> None:
        super().__init__(mes_config, qkv_bias=True, qk_norm=False)


class DecoderModel(nn.Module):
    """``Qwen2Model`` / ``Qwen3Model`` (``qwen2.py:168-192``, ``qwen3.py:142-166``)."""

    layer_cls = Qwen2DecoderLayer

    def __init__(self, mes_config: MESConfig) -> None:
        super().__init__()
        self.mes_config = mes_config
        mc = mes_config.model_config
        self.embed_tokens = VocabParallelEmbedding(mc.vocab_size, mc.hidden_size)
        self.layers = nn.ModuleList([self.layer_cls(mes_config)
                                     for _ in range(mc.num_hidden_layers)])
        self.norm = RMSNorm(mc.hidden_size, eps=mc.rms_norm_eps)
        # The tensor-parallel group size the layers were sharded for (fixed here: a process
        # group created later - e.g. for data-parallel replicas - does not shard the model).
        self.tp_size = _tp_size()

    # Tensor parallelism: below this many tokens the batch is not split for overlap.
    overlap_min_tokens = int(os.environ.get("MES_TP_OVERLAP_MIN_TOKENS", "4096"))
    # Neither micro-batch may have 256 tokens or fewer: the GEMMs split K over clusters for
    # such batches, which rounds differently from the whole batch's kernels, and the
    # overlapped forward must equal the unsplit one bit for bit.
    overlap_min_part = 257
    @staticmethod
    def overlap_reserved_sms(world_size: int) -> int:
        """SMs kept free of the persistent kernels while all-reduces overlap them: the NCCL
        kernels' share (callers cap NCCL at as many channels).  More GPUs leave each one
        less compute to hide the collectives behind, so the collectives get more SMs:
        16 at 2 GPUs (measured best at TP2), 24 at 4, 32 at 8.  MES_TP_RESERVED_SMS
        overrides."""
        env = os.environ.get("MES_TP_RESERVED_SMS")
        if env is not None:
            return int(env)
        return 16 if world_size <= 2 else 24 if world_size <= 4 else 32

    # overlap_split value meaning "the host found no valid micro-batch boundary".
    NO_SPLIT = -1

    def _resolve_split(self, positions: torch.Tensor, overlap_split: int | None) -> int | None:
        """The micro-batch boundary to use, or None for the unsplit forward.  A boundary the
        caller worked out from the host copy of the batch (:meth:`overlap_split_host`; a
        negative value when there is none) is taken as given - inside a CUDA-graph capture
        no device read may happen; only ``None`` (not given) derives it from ``positions``
        with one device synchronisation."""
        if self.tp_size == 1:
            return None
        if overlap_split is None:
            return self._overlap_split(positions)
        return int(overlap_split) if overlap_split >= 0 else None

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor,
                overlap_split: int | None = None) -> torch.Tensor:
        """``overlap_split``: at tp > 1, the micro-batch boundary (a sequence start) when the
        caller knows it from the host copy of the batch (see :meth:`overlap_split_host`,
        ``NO_SPLIT`` when there is none); ``None`` derives it from ``positions``."""
        split = self._resolve_split(positions, overlap_split)
        if split is not None:
            return self._forward_overlapped(input_ids, positions, split)
        with batch_schedule(positions):
            hidden_states = self.embed_tokens.forward_f32(input_ids)
            residual = None
            for layer in self.layers:
                hidden_states, residual = layer(positions, hidden_states, residual)
            return self.norm.residual_norm(residual, hidden_states)

    def forward_last_rows(self, input_ids: torch.Tensor, positions: torch.Tensor,
                          rows: torch.Tensor) -> torch.Tensor:
        """Final hidden states ``[B, H]`` of the token rows ``rows`` (int64 [B]) only - the
        rows the embedding post-process pools (``core/gpu_worker.py:258``).  Every layer
        but the last runs on all tokens; the last runs its o_proj, MLP and final norm on
        the B rows (:meth:`DecoderLayer.forward_last_rows`).  Each returned row equals the
        corresponding row of :meth:`forward`.  Unsplit forward only (tp == 1, or a batch
        the tensor-parallel overlap does not split)."""
        with batch_schedule(positions):
            hidden_states = self.embed_tokens.forward_f32(input_ids)
            residual = None
            for layer in self.layers[:-1]:
                hidden_states, residual = layer(positions, hidden_states, residual)
            delta, res = self.layers[-1].forward_last_rows(positions, hidden_states, residual, rows)
            return self.norm.residual_norm(res, delta)

    def _overlap_split(self, positions: torch.Tensor) -> int | None:
        """Token index of the sequence start nearest the middle of the batch, or None when
        the forward runs unsplit (tp == 1, a small batch, or a single sequence)."""
        T = positions.shape[0]
        if self.tp_size == 1 or T < self.overlap_min_tokens:
            return None
        starts = (torch.nonzero(positions[1:] != positions[:-1] + 1).flatten() + 1).cpu()
        return self._nearest_middle(starts.numpy(), T)

    @classmethod
    def overlap_split_host(cls, positions, tp_size: int | None = None) -> int:
        """:meth:`_overlap_split` from a host (numpy) copy of ``positions`` for a model
        sharded ``tp_size`` ways (default: the current process group's size);
        ``NO_SPLIT`` when the forward runs unsplit."""
        import numpy as np
        pos = np.asarray(positions)
        T = pos.shape[0]
        tp = _tp_size() if tp_size is None else tp_size
        if tp == 1 or T < cls.overlap_min_tokens:
            return cls.NO_SPLIT
        split = cls._nearest_middle(np.flatnonzero(pos[1:] != pos[:-1] + 1) + 1, T)
        return cls.NO_SPLIT if split is None else split

    @classmethod
    def _nearest_middle(cls, starts, T: int) -> int | None:
        import numpy as np
        starts = np.asarray(starts)
        starts = starts[(starts >= cls.overlap_min_part) & (T - starts >= cls.overlap_min_part)]
        if len(starts) == 0:
            return None
        return int(starts[np.argmin(np.abs(starts - T // 2))])

    def _forward_overlapped(self, input_ids, positions, split: int) -> torch.Tensor:
        """Tensor-parallel forward as two micro-batches of whole sequences, A = tokens
        [0, split) and B = [split, T), interleaved per half-block on the compute stream:
        A's attention, B's attention, A's MLP, B's MLP, ...  Each half-block ends in an
        asynchronous all-reduce of its partial product, which runs while the other
        micro-batch computes; the next half-block of the same micro-batch waits for it on
        the stream (no host synchronisation).  Per token the arithmetic is the unsplit
        forward's."""
        T = positions.shape[0]
        parts = ((0, split), (split, T))
        pos = [positions[a:b] for a, b in parts]
        _C.set_sm_reserve(self.overlap_reserved_sms(self.tp_size))
        try:
            with batch_schedule(pos[0]), batch_schedule(pos[1]):
                residual = self.embed_tokens.forward_f32(input_ids)
                res = [residual[a:b] for a, b in parts]
                pending = [None, None]

                def norm_after(norm, m, out=None):
                    if pending[m] is None:
                        return norm.residual_norm(res[m], None, out)
                    delta, work = pending[m]
                    work.wait()
                    return norm.residual_norm(res[m], delta, out)

                for layer in self.layers:
                    layer.build_panels(min(split, T - split))
                    for m in (0, 1):
                        x = norm_after(layer.input_layernorm, m)
                        y = layer.self_attn.forward_partial(pos[m], x)
                        pending[m] = (y, dist.all_reduce(y, async_op=True))
                    for m in (0, 1):
                        x = norm_after(layer.post_attention_layernorm, m)
                        y = layer.mlp.forward_partial(x)
                        pending[m] = (y, dist.all_reduce(y, async_op=True))
                    layer.clear_panels()
                out = torch.empty(T, residual.shape[1], dtype=torch.bfloat16,
                                  device=residual.device)
                for m, (a, b) in enumerate(parts):
                    norm_after(self.norm, m, out[a:b])
                return out
        finally:
            _C.set_sm_reserve(0)


class Qwen2Model(DecoderModel):
    layer_cls = Qwen2DecoderLayer


class CausalLMBase(nn.Module):
    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", 0),
        "up_proj": ("gate_up_proj", 1),
    }
    model_cls = Qwen2Model

    def __init__(self, mes_config: MESConfig = None) -> None:
        super().__init__()
        if mes_config is None:
            mes_config = MESConfig()
        self.mes_config = mes_config
        self.model = self.model_cls(mes_config)

    @property
    def tp_size(self) -> int:
        return self.model.tp_size

    def process_weights_after_loading(self):
        """Repack every AWQ weight into the kernel layout (once, after loading)."""
        for m in self.modules():
            if hasattr(m, "qweight") and hasattr(m, "process_weights_after_loading") and m is not self:
                m.process_weights_after_loading()

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor,
                overlap_split: int | None = None) -> torch.Tensor:
        return self.model(input_ids, positions, overlap_split)

    def forward_last_rows(self, input_ids: torch.Tensor, positions: torch.Tensor,
                          rows: torch.Tensor) -> torch.Tensor:
        return self.model.forward_last_rows(input_ids, positions, rows)


@register_model("Qwen2ForCausalLM")
class Qwen2ForCausalLM(CausalLMBase):
    model_cls = Qwen2Model
