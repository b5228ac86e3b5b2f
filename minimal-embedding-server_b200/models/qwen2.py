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

import torch
import torch.distributed as dist
from torch import nn

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

    def forward_residual(self, x, residual):
        if self.gate_up_proj.supports_silu():
            act = self.gate_up_proj.forward_silu(x)   # GEMM with SiLU-and-mul epilogue
        else:
            act = self.act_fn(self.gate_up_proj(x))
        return self.down_proj.forward_residual(act, residual)


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

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor | None,
                residual: torch.Tensor | None):
        """One block on the fp32 residual stream.  First layer: ``hidden_states`` is the
        fp32 embedding, which becomes the residual.  Later layers: ``hidden_states`` is the
        previous block's pending delta (None once it was added in a GEMM epilogue)."""
        if residual is None:
            residual = hidden_states
            x = self.input_layernorm.residual_norm(residual)
        else:
            x = self.input_layernorm.residual_norm(residual, hidden_states)
        delta = self.self_attn.forward_residual(positions, x, residual)
        x = self.post_attention_layernorm.residual_norm(residual, delta)
        delta = self.mlp.forward_residual(x, residual)
        return delta, residual


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

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        with batch_schedule(positions):
            hidden_states = self.embed_tokens.forward_f32(input_ids)
            residual = None
            for layer in self.layers:
                hidden_states, residual = layer(positions, hidden_states, residual)
            return self.norm.residual_norm(residual, hidden_states)


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

    def process_weights_after_loading(self):
        """Repack every AWQ weight into the kernel layout (once, after loading)."""
        for m in self.modules():
            if hasattr(m, "qweight") and hasattr(m, "process_weights_after_loading") and m is not self:
                m.process_weights_after_loading()

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids, positions)


@register_model("Qwen2ForCausalLM")
class Qwen2ForCausalLM(CausalLMBase):
    model_cls = Qwen2Model
