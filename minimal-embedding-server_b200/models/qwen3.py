"""Qwen3 decoder (``models/qwen3.py``): Qwen2's block plus per-head q/k RMSNorm before
RoPE (``qwen3.py:82-88``), fused with the rotation into one kernel, and the QKV bias
taken from ``attention_bias`` (``:117``)."""
from __future__ import annotations

from ..schemas.config import MESConfig
from .qwen2 import CausalLMBase, DecoderLayer, DecoderModel
from .registry import register_model


class Qwen3DecoderLayer(DecoderLayer):

    def __init__(self, mes_config: MESConfig) -> None:
        super().__init__(mes_config,
                         qkv_bias=bool(getattr(mes_config.model_config, "attention_bias", False)),
                         qk_norm=True)


class Qwen3Model(DecoderModel):
    layer_cls = Qwen3DecoderLayer


@register_model("Qwen3ForCausalLM")
class Qwen3ForCausalLM(CausalLMBase):
    model_cls = Qwen3Model
