"""``MESConfig`` (``schemas/config.py:1-16``) plus the AWQ quantisation settings."""
from __future__ import annotations


class MESConfig:
    def __init__(self, attn_backend: str = "b200", model_name: str | None = None,
                 max_tokens_per_batch: int | None = None, enable_monitoring: bool | None = None,
                 dtype: str = "auto", model_config=None, quant_config=None):
        self.attn_backend = attn_backend
        self.model_name = model_name
        self.max_tokens_per_batch = max_tokens_per_batch
        self.enable_monitoring = enable_monitoring
        self.dtype = dtype
        self.model_config = model_config
        if quant_config is None:
            from ..layers.linear import AWQConfig
            qc = getattr(model_config, "quantization_config", None) if model_config else None
            if isinstance(qc, dict) and qc.get("quant_method", "awq") != "awq":
                raise ValueError(f"unsupported quantization method {qc.get('quant_method')}")
            group = qc.get("group_size", 128) if isinstance(qc, dict) else 128
            bits = qc.get("bits", qc.get("w_bit", 4)) if isinstance(qc, dict) else 4
            quant_config = AWQConfig(group_size=group, bits=bits)
        self.quant_config = quant_config
