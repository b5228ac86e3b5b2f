"""Attention layers package (``layers/attention/__init__.py``)."""
from .b200 import B200Attention, batch_schedule
from .base import BaseAttention, create_attention

__all__ = ["BaseAttention", "create_attention", "B200Attention", "batch_schedule"]
