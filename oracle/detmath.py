"""Deterministic scalar arithmetic shared, operation for operation, by the CPU oracle and the
CUDA kernels (``fleet-amd-task_b200/csrc/detmath.cuh`` is the device twin of this file).

TEST INFRASTRUCTURE. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import anything under ``oracle/``.

Why this file exists. The reference's NumPy specification (harness/numpy_ref.py:36-321)
leaves two things open: the summation order of every FP32 dot product ("the summation order
is not specified", numpy_ref.py:18-20) and the implementation of exp/log. Both make a CPU
oracle and a GPU kernel disagree in the last bit, and a last-bit difference in a BF16
rounding can flip a router choice or a greedy token. This restatement closes both:

* every dot product of BF16 values is computed exactly (the products are exact in FP64 and
  the FP64 sum of at most a few thousand of them is exact to 2^-53) and rounded ONCE, to
  FP32 or straight to BF16; the kernels accumulate in FP64 too, so any summation order gives
  the same rounded value (they differ only if the exact sum lies within ~1e-16 relative of a
  rounding midpoint);
* exp and log are the two routines below, made of separately rounded FP32 operations (no
  fused multiply-add), which IEEE-754 makes bit-identical on any machine. The kernels use
  ``__fmul_rn``/``__fadd_rn``/``__fsub_rn``/``__fdiv_rn``, which the compiler never contracts.

Methods (published, restated here from the mathematics):
* exp: Cody & Waite argument reduction (W. J. Cody, W. Waite, "Software Manual for the
  Elementary Functions", 1980): x = k ln2 + r with ln2 split in a 16-bit head and a tail so
  k * head is exact, |r| <= ln2/2; exp(r) by its Taylor series to degree 7 (remainder
  < 6e-9 relative) in Horner form; the result scaled by 2^k through the exponent field.
* log: m = x / 2^e in [sqrt(1/2), sqrt(2)), log m = 2 atanh(t), t = (m-1)/(m+1), by the series
  2t (1 + t^2/3 + t^4/5 + t^6/7 + t^8/9) (Abramowitz & Stegun 4.1.27; |t| <= 0.1716 so the
  remainder is < 3e-9 relative), plus e ln2 with the same split of ln2.
"""
import math

import numpy as np

F32 = np.float32
F64 = np.float64

# ---------------------------------------------------------------------------------------------
# constants, derived from the mathematics (not copied from any library)

LOG2E = F32(1.0 / math.log(2.0))
LN2_HI = F32(round(math.log(2.0) * 65536.0) / 65536.0)       # 45426 / 65536: 16 significant bits
LN2_LO = F32(math.log(2.0) - float(LN2_HI))
EXP_C = [F32(1.0 / math.factorial(n)) for n in range(8)]      # Taylor coefficients of exp
LOG_C = [F32(1.0 / n) for n in (1, 3, 5, 7, 9)]               # atanh series coefficients
SQRT2 = F32(math.sqrt(2.0))
EXP_LO = F32(-87.0)      # below: result 0 (true value < 2^-125, flushed)
EXP_HI = F32(88.0)       # above: +inf (true value > 1.6e38)

# the exponent field offsets of the FP64 "bit placement" trick used by the kernels to turn a
# BF16 pattern into an FP64 scaled by 2^-896 without a conversion instruction; the activation
# operand is pre-scaled by 2^832 so every product carries 2^-64, undone once per dot product
BF16_F64_SHIFT = 45
W_SCALE_LOG2 = -896
X_SCALE_LOG2 = 832
DOT_UNSCALE_LOG2 = 64


def _f32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=F32))


# ---------------------------------------------------------------------------------------------
# BF16 rounding


def bf16(x):
    """Round FP32 values to BF16 precision (round to nearest even); returns float32 values.
    Same bit arithmetic as harness/numpy_ref.py:36-42 (bf16)."""
    x = _f32(x)
    u = x.view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    u = (u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)
    return u.view(F32)


def bf16_from_f64(x):
    """Round FP64 values straight to BF16 (one rounding, nearest even); returns float32 values.

    Normal BF16 range: add the rounding bias at bit 45 of the FP64 pattern (52 - 7 mantissa
    bits) and clear the bits below; the result has 8 significant bits and converts to FP32
    exactly (or overflows to inf exactly as a BF16 would). Below 2^-126 (BF16 subnormals) the
    value is rounded on the 2^-133 grid instead. NaN stays NaN."""
    x = np.ascontiguousarray(np.asarray(x, dtype=F64))
    u = x.view(np.uint64)
    lsb = (u >> np.uint64(45)) & np.uint64(1)
    r = (u + np.uint64((1 << 44) - 1) + lsb) & ~np.uint64((1 << 45) - 1)
    out = r.view(F64)
    tiny = np.abs(x) < 2.0 ** -126
    if tiny.any():
        out = np.where(tiny, np.rint(x * 2.0 ** 133) * 2.0 ** -133, out)
    out = np.where(np.isnan(x), np.nan, out)
    with np.errstate(over="ignore"):
        return out.astype(F32)


def f32_from_f64(x):
    """FP64 -> FP32, round to nearest even (the IEEE conversion; __double2float_rn)."""
    return np.asarray(x, dtype=F64).astype(F32)


def bf16_bits(x):
    """BF16 values (as float32) -> their uint16 patterns."""
    return (_f32(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(b):
    """uint16 BF16 patterns -> float32 values."""
    return (np.asarray(b, dtype=np.uint32) << np.uint32(16)).view(F32)


# ---------------------------------------------------------------------------------------------
# exact dot products


def dot_exact(W, x):
    """Rows of W (BF16 values) against x (BF16 or FP32 values), every product exact, summed in
    FP64. Returns FP64; the caller rounds once (bf16_from_f64 or f32_from_f64)."""
    return np.asarray(W, F64) @ np.asarray(x, F64)


def sum_f64(x, axis=-1):
    return np.sum(np.asarray(x, F64), axis=axis)


# ---------------------------------------------------------------------------------------------
# exp and log


def det_exp(x):
    """exp(x) in FP32 by Cody-Waite reduction and a degree-7 Taylor polynomial, every step a
    separately rounded FP32 operation. x < -87 gives 0, x > 88 gives +inf, NaN stays NaN.
    Maximum error against the exact value: under 2 FP32 ulp (tests/test_oracle_detmath.py)."""
    x = _f32(x)
    with np.errstate(invalid="ignore", over="ignore"):
        xc = np.clip(np.nan_to_num(x, nan=0.0), EXP_LO, EXP_HI).astype(F32)
        k = np.rint(xc * LOG2E).astype(F32)
        r = ((xc - k * LN2_HI).astype(F32) - (k * LN2_LO).astype(F32)).astype(F32)
        p = EXP_C[7]
        for n in range(6, -1, -1):
            p = (p * r).astype(F32) + EXP_C[n]
            p = p.astype(F32)
        scale = ((k.astype(np.int32) + np.int32(127)) << np.int32(23)).astype(np.int32).view(F32)
        y = (p * scale).astype(F32)
    y = np.where(x < EXP_LO, F32(0.0), y)
    y = np.where(x > EXP_HI, F32(np.inf), y)
    y = np.where(np.isnan(x), F32(np.nan), y)
    return y.astype(F32)


def det_log(x):
    """Natural log in FP32 (atanh series on the mantissa, exponent times ln2), every step a
    separately rounded FP32 operation. 0 -> -inf, negative or NaN -> NaN, +inf -> +inf.
    Maximum error against the exact value: under 3 FP32 ulp for x > 0 (worst near x = 1)."""
    x = _f32(x)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        xs = np.where((x > 0) & (x < F32(2.0 ** -126)), (x * F32(2.0 ** 24)).astype(F32), x).astype(F32)
        esub = np.where((x > 0) & (x < F32(2.0 ** -126)), np.int32(24), np.int32(0))
        bits = np.abs(xs).view(np.uint32)
        e = ((bits >> np.uint32(23)).astype(np.int32) - np.int32(127)) - esub
        m = ((bits & np.uint32(0x7FFFFF)) | np.uint32(0x3F800000)).view(F32)
        big = m > SQRT2
        m = np.where(big, (m * F32(0.5)).astype(F32), m).astype(F32)
        e = np.where(big, e + 1, e)
        t = ((m - F32(1.0)).astype(F32) / (m + F32(1.0)).astype(F32)).astype(F32)
        t2 = (t * t).astype(F32)
        s = LOG_C[4]
        for c in (LOG_C[3], LOG_C[2], LOG_C[1], LOG_C[0]):
            s = ((s * t2).astype(F32) + c).astype(F32)
        logm = ((t + t).astype(F32) * s).astype(F32)
        ef = e.astype(F32)
        y = ((ef * LN2_HI).astype(F32) + ((ef * LN2_LO).astype(F32) + logm).astype(F32)).astype(F32)
    y = np.where(x == 0, F32(-np.inf), y)
    y = np.where(x == np.inf, F32(np.inf), y)
    y = np.where((x < 0) | np.isnan(x), F32(np.nan), y)
    return y.astype(F32)


def silu(x):
    """SiLU in FP32: x / (1 + det_exp(-x)), an IEEE division (numpy_ref.py:248-253 restated
    with the deterministic exp; the reference's kernels use a fast exp and reciprocal there)."""
    x = _f32(x)
    with np.errstate(over="ignore"):
        return (x / (F32(1.0) + det_exp(-x)).astype(F32)).astype(F32)
