"""B200 (sm_100a) FP8 attention / FP8 linear hot path for MiniMax-H3.

Layout:
  csrc/        CUDA kernels (tcgen05 / TMA) and the C ABI of libmh3_b200.so
  _lib.py      ctypes binding of that ABI (include/mh3_b200.h)
  ops.py       torch-facing wrappers (pointers, strides, streams)
  kernels/     drop-in mirror of the reference's ``kernels`` package
               (fp8_attention, attention_router, fp8_linear) and the fused
               LoRA wrapper of unquantised linears (lora)
  streaming.py fp8_attention over host-resident tensors
  ulysses.py   head-parallel (Ulysses) sharding over NCCL
  build.py     nvcc recipe that builds libmh3_b200.so in-tree
"""
__version__ = "0.1.0"
