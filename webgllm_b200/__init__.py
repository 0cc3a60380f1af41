"""webgllm_b200: webgllm's 4-bit matmul path, B200-native.

The product is libwebgllm_b200.so (include/webgllm_q4.h); ``q4`` mirrors the
reference's interface for the path (src/repack.ts, src/engine.ts matmul
entry points) on top of it.
"""
from .q4 import (  # noqa: F401
    Context, GpuError, QuantMatrix, RangeError, ShapeError, context, matmul, matrixRow,
    newQuantMatrix, packMatMulNBits, packQ4_0, project, writeMatrix,
)
