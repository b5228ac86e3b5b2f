"""Layers with the reference's interfaces (``layers/``), computed by sm_100a kernels."""
