"""mes_b200 - B200 (sm_100a) engine for the embedding server's GPU-worker forward pass.

A packed variable-length batch of token ids runs through a Qwen3 / Qwen2 decoder with AWQ
int4 weights and ends in last-token pooling + L2 normalisation.  The layer and model API
mirrors the reference server (``layers/``, ``models/``, ``core/gpu_worker.py``); all math
runs in hand-written CUDA kernels for sm_100a behind the C ABI of ``include/mes_b200.h``
(``lib/libmes_b200.so``, loaded by ``_C``).
"""
__version__ = "0.1.0"

from . import _C  # noqa: F401
