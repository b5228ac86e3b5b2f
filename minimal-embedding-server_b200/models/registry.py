"""Architecture name -> model class (``models/registry.py:1-25``)."""
from __future__ import annotations

from typing import Dict, Type

MODEL_REGISTRY: Dict[str, Type] = {}


def register_model(architecture: str):
    def decorator(model_class):
        MODEL_REGISTRY[architecture] = model_class
        return model_class
    return decorator


def get_model_class(config):
    if not getattr(config, "architectures", None):
        raise ValueError("Model config does not have 'architectures' field")
    architecture = config.architectures[0]
    if architecture not in MODEL_REGISTRY:
        raise ValueError(f"Unsupported model architecture: {architecture}. "
                         f"Available architectures: {list(MODEL_REGISTRY)}")
    return MODEL_REGISTRY[architecture]
