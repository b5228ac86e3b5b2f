"""CPU oracle for the embedding forward pass (test infrastructure only).

This package restates, on the CPU, what the reference (woodx9/minimal-embedding-server)
computes on the GPU-worker hot path, so that the CUDA kernels of ``mes_b200`` can be
checked against it.  It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may import it.
The product path (``mes_b200``) never imports this package and has no CPU fallback.

Modules
-------
``awq``    numpy restatement of the AWQ int4 storage format (AutoAWQ "GEMM" packing
           order, pinned against vLLM's ``awq_pack``) and of the exact dequantisation
           ``w = (q - z) * s``; plus the kernel-side repacked layout.
``ops``    torch-CPU fp32 restatements of the per-op arithmetic in the reference's
           ``layers/`` (RMSNorm, fused add+RMSNorm, NeoX RoPE, SiLU-and-mul, varlen causal
           GQA attention, vocab embedding, last-token pooling + L2 normalisation).
``model``  the Qwen3 / Qwen2 decoder forward of ``models/qwen3.py`` / ``models/qwen2.py``
           built from ``ops``, with dense or AWQ-dequantised weights and optional
           tensor-parallel sharding over a ``gloo`` process group.

Parity pinning
--------------
* ``ops`` and ``model`` are pinned against outputs of the reference's own Python model
  code run on CPU (fixtures in ``tests/golden/`` written by
  ``tests/golden/make_golden.py``).
* ``awq`` packing order is pinned against vLLM 0.22.0's ``awq_pack`` (fixture written by
  the same script).  The reference itself contains no AWQ code, so the dequantised
  *values* are defined here (exact fp32 product, one round-to-nearest-even to bf16) and
  are "parity unpinned" with respect to the reference.
"""
