"""Stated tolerances for the parity tests, per precision path.

normwise  max|got - ref| / max|ref|
floored   max over elements of |got - ref| / max(|ref|, 1e-3 max|ref|)

fp32: fp32 CUDA-core arithmetic. The reference itself (fp32/complex64) is ~1e-6 normwise and up
      to ~4e-4 floored against the exact recurrence, so the fp32 path is held to 2e-5 normwise
      and 2e-3 floored against the reference and against the fp64 recurrence.
tf32: tensor-core tiles with tf32 operands (10-bit mantissa); the bar is 2e-2.
"""

TOL = {
    "fp32": {"y_normwise": 2e-5, "y_floored": 2e-3, "g_normwise": 5e-5},
    "tf32": {"y_normwise": 2e-2, "y_floored": 2e-2, "g_normwise": 2e-2},
}
