"""CPU oracle for the MiniMax-H3 FP8 attention / FP8 linear hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
directory: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline arm use it, and only as the checker (or as the timed CPU
reference), never as the thing measured on the GPU.

Contents
--------
``fp8_attention_ref``
    A vectorised torch-on-CPU restatement of the reference's
    ``kernels/fp8_attention.py`` (quantise Q / K / V, the flash-attention
    kernel with its bit-trick P, lazy max and optional repair), plus the
    fp32 SDPA oracle on dequantised inputs that the north-star tolerance is
    stated against, plus an emulation of this package's own exp2 softmax.
``fp8_linear_ref``
    Restatement of ``kernels/fp8_linear.py``: per-row e4m3 quantisation, the
    row-wise scaled GEMM that ``torch._scaled_mm`` computes, and the LoRA
    adapter epilogue.
``router_ref``
    The reference's CPU path for this hot path: ``routed_sdpa`` falling back
    to torch's SDPA on CPU tensors (``kernels/attention_router.py:93-102``).

Parity pin
----------
The restatement is pinned against golden vectors in ``tests/golden/`` that
were produced by running the reference's own Triton kernels (unmodified) under
Triton's CPU interpreter, with only the interpreter's faulty numeric
conversion helper replaced by correctly rounded casts; see
``tests/golden/make_golden.py``.  ``torch._scaled_mm`` (a library GEMM) has no
CPU implementation for row-wise scales, so the GEMM itself is restated from
its documented semantics and is pinned only through the quantisation and
LoRA pieces that do run.
"""
