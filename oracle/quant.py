"""Per-row symmetric INT8 quantiser -- TEST INFRASTRUCTURE ONLY (the checker).

numpy restatement of the reference's ``quantize_kernel``
(visheshnarayan/llm.cu src/kernels/quantize.cu:8-50), term by term in fp32:

* absmax = max |w| over the row (fp32)                        quantize.cu:17-34
* scale  = absmax / 127.0f     (IEEE division, no fast-math)  quantize.cu:36
* inv    = scale > 0 ? 1.0f / scale : 0.0f                    quantize.cu:41
* q      = (int8) rintf(fminf(fmaxf(w * inv, -127), 127))     quantize.cu:42-47
  rintf rounds half to even, as does numpy's ``rint``.

The reference is built without ``--use_fast_math`` and each step is a single
correctly-rounded fp32 operation, so a CUDA implementation that performs the
same operations in the same order is bit-exact with this function.

``dequant_gemm_nt`` restates ``matmul_int8_kernel`` (quantize.cu:55-70):
C = (A . q^T) * scale[n], the scale applied once in the epilogue.
"""
from __future__ import annotations

import numpy as np


def quantize_rows(w: np.ndarray):
    """w fp32 [rows, cols] -> (q int8 [rows, cols], scale fp32 [rows])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    absmax = np.max(np.abs(w), axis=1).astype(np.float32) if w.shape[1] else np.zeros(w.shape[0], np.float32)
    scale = (absmax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(scale > 0, np.float32(1.0) / scale, np.float32(0.0)).astype(np.float32)
    val = (w * inv[:, None]).astype(np.float32)
    val = np.minimum(np.maximum(val, np.float32(-127.0)), np.float32(127.0))
    q = np.rint(val).astype(np.int8)
    return q, scale


def dequant_gemm_nt(a: np.ndarray, q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """C[M, N] = (A[M, K] . q[N, K]^T) * scale[N] in float64 accumulation."""
    acc = np.asarray(a, np.float64) @ np.asarray(q, np.float64).T
    return (acc * np.asarray(scale, np.float64)[None, :]).astype(np.float32)
