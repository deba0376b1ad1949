"""NumPy-named ufuncs (mirrors ``src/macmetalpy/ufunc_ops.py``).

Each builds a lazy fused node with numpy's type resolution.  Differences
from the reference at scale (its GPU path) are on purpose, to match its CPU
path (numpy): integer ``floor_divide`` floors (the MSL kernel truncates,
``_kernels.py:44``); ``fmod`` computes fmod (``ufunc_ops.fmod`` dispatches
``hypot_op`` above the threshold); ``divide`` of integers gives numpy's
float64 (resolved by ``float64_behavior``) instead of a hard float32.
"""

from __future__ import annotations

from .math_ops import _b, _u

__all__ = [
    "add", "subtract", "multiply", "divide", "true_divide", "floor_divide", "float_power", "fmod",
    "hypot", "arctan2", "logaddexp", "logaddexp2", "heaviside", "copysign", "nextafter", "fmax", "fmin",
    "maximum", "minimum", "exp2", "expm1", "log1p", "cbrt", "reciprocal", "rint", "trunc", "fix",
    "arcsinh", "arccosh", "arctanh", "degrees", "radians", "rad2deg", "deg2rad", "less", "less_equal",
    "greater", "greater_equal", "equal", "not_equal",
]

add = _b("add_op")
subtract = _b("sub_op")
multiply = _b("mul_op")
divide = _b("div_op")
true_divide = divide
floor_divide = _b("floor_divide_op")
fmod = _b("fmod_op")
hypot = _b("hypot_op")
arctan2 = _b("atan2_op")
logaddexp = _b("logaddexp_op")
logaddexp2 = _b("logaddexp2_op")
heaviside = _b("heaviside_op")
copysign = _b("copysign_op")
nextafter = _b("nextafter_op")
fmax = _b("fmax_op")
fmin = _b("fmin_op")
maximum = _b("max_op")
minimum = _b("min_op")
less = _b("lt_op")
less_equal = _b("le_op")
greater = _b("gt_op")
greater_equal = _b("ge_op")
equal = _b("eq_op")
not_equal = _b("ne_op")
exp2 = _u("exp2_op")
expm1 = _u("expm1_op")
log1p = _u("log1p_op")
cbrt = _u("cbrt_op")
reciprocal = _u("reciprocal_op")
rint = _u("rint_op")
trunc = _u("trunc_op")
fix = trunc
arcsinh = _u("asinh_op")
arccosh = _u("acosh_op")
arctanh = _u("atanh_op")
degrees = _u("degrees_op")
rad2deg = degrees
radians = _u("radians_op")
deg2rad = radians


def float_power(x1, x2, **kwargs):
    from .creation import asarray
    return _b("pow_op")(asarray(x1).astype("float64"), x2)
