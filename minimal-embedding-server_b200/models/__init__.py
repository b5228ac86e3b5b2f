"""Model classes; importing registers them (``models/__init__.py``)."""
from .qwen2 import Qwen2ForCausalLM
from .qwen3 import Qwen3ForCausalLM
from .registry import MODEL_REGISTRY, get_model_class, register_model

__all__ = ["Qwen2ForCausalLM", "Qwen3ForCausalLM", "MODEL_REGISTRY", "get_model_class",
           "register_model"]
