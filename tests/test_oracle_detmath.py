"""The oracle's deterministic arithmetic: BF16 rounding against torch, the straight FP64->BF16
rounding against exact rational rounding, and det_exp / det_log against FP64 error bounds."""
import math
from fractions import Fraction

import numpy as np
import pytest
import torch

from oracle import detmath as D


def ulp_err(got, exact):
    """|got - exact| in FP32 ulps of the exact value (FP64 exact)."""
    exact = np.asarray(exact, np.float64)
    got = np.asarray(got, np.float64)
    e = np.floor(np.log2(np.maximum(np.abs(exact), 2.0 ** -126)))
    ulp = 2.0 ** (e - 23)
    return np.abs(got - exact) / ulp


def test_bf16_matches_torch():
    xs = np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 100
    xs = np.concatenate([xs, np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5e-3, 65504.0, 0.0, -0.0], np.float32)])
    assert np.array_equal(D.bf16(xs), torch.tensor(xs).bfloat16().float().numpy())


def _bf16_exact_round(v):
    """Round a Fraction to the nearest BF16 (ties to even), normal range."""
    if v == 0:
        return 0.0
    s = -1 if v < 0 else 1
    a = abs(v)
    e = math.floor(math.log2(a))
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    q = a / Fraction(2) ** (e - 7)               # 8 significant bits
    n = math.floor(q)
    r = q - n
    if r > Fraction(1, 2) or (r == Fraction(1, 2) and n % 2 == 1):
        n += 1
    return s * float(n * Fraction(2) ** (e - 7))


def test_bf16_from_f64_is_one_rounding():
    rng = np.random.default_rng(1)
    xs = rng.standard_normal(3000) * np.exp(rng.uniform(-20, 20, 3000))
    # values that a double rounding through FP32 would get wrong: just above a BF16 midpoint
    mids = np.array([1.0 + 2 ** -8 + 2 ** -40, 1.0 + 2 ** -8 - 2 ** -40, -(3.0 + 2 ** -7 + 2 ** -35)])
    xs = np.concatenate([xs, mids])
    got = D.bf16_from_f64(xs)
    want = np.array([_bf16_exact_round(Fraction(float(x))) for x in xs], np.float32)
    assert np.array_equal(got, want)
    # an FP32 detour would round 1 + 2^-8 + 2^-40 to the midpoint and then to even (1.0)
    assert D.bf16_from_f64(np.array([1.0 + 2 ** -8 + 2 ** -40]))[0] == np.float32(1.0 + 2 ** -7)


def test_bf16_from_f64_subnormal_and_specials():
    xs = np.array([2.0 ** -130, -3 * 2.0 ** -134, np.inf, -np.inf, 3.5e38, np.nan])
    got = D.bf16_from_f64(xs)
    assert got[0] == np.float32(2.0 ** -130)
    assert got[1] == np.float32(-2.0 ** -132)        # 1.5 ulp of the 2^-133 grid -> 2 (even)
    assert got[2] == np.inf and got[3] == -np.inf and got[4] == np.inf and np.isnan(got[5])


def test_det_exp_error_bound():
    rng = np.random.default_rng(2)
    xs = np.concatenate([rng.uniform(-87, 88, 200000), rng.uniform(-1, 1, 50000),
                         np.array([0.0, -0.0, 1e-30, -1e-30, 88.0, -87.0])]).astype(np.float32)
    got = D.det_exp(xs)
    exact = np.exp(xs.astype(np.float64))
    assert got.dtype == np.float32
    normal = exact >= 2.0 ** -126
    assert ulp_err(got[normal], exact[normal]).max() < 2.0
    assert D.det_exp(np.float32(0.0)) == 1.0
    sp = D.det_exp(np.array([-np.inf, -100.0, 100.0, np.inf, np.nan], np.float32))
    assert sp[0] == 0 and sp[1] == 0 and sp[2] == np.inf and sp[3] == np.inf and np.isnan(sp[4])


def test_det_log_error_bound():
    rng = np.random.default_rng(3)
    xs = np.concatenate([np.exp(rng.uniform(-80, 80, 200000)), rng.uniform(0.5, 2.0, 50000),
                         rng.uniform(1.0, 64.0, 50000), np.array([1.0, 2.0, 1e-40, 3e-45])]).astype(np.float32)
    xs = xs[xs > 0]
    got = D.det_log(xs)
    exact = np.log(xs.astype(np.float64))
    err = np.abs(got.astype(np.float64) - exact)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 2.0 ** -126))) - 23)
    # worst near x = 1 (e = 0), where the rounding of m + 1 and of the quotient dominate
    assert (err / ulp).max() < 3.0
    assert D.det_log(np.float32(1.0)) == 0.0
    sp = D.det_log(np.array([0.0, -1.0, np.inf, np.nan], np.float32))
    assert sp[0] == -np.inf and np.isnan(sp[1]) and sp[2] == np.inf and np.isnan(sp[3])


def test_silu_close_to_exact():
    xs = np.random.default_rng(4).uniform(-30, 30, 100000).astype(np.float32)
    got = D.silu(xs).astype(np.float64)
    x64 = xs.astype(np.float64)
    exact = x64 / (1.0 + np.exp(-x64))
    assert np.all(np.abs(got - exact) <= 4 * np.abs(exact) * 2.0 ** -24 + 1e-37)


def _scalar_row_dot(w, x):
    """The kernels' row-dot order spelled out one FP32 operation at a time."""
    K = len(x)
    ks, kp, maxv = D.gemv_parts(K)
    parts = []
    for p in range(ks):
        lanes = []
        for l in range(32):
            a0, a1 = np.float32(0), np.float32(0)
            for j in range(maxv):
                v = l + 32 * j
                if v * 8 >= kp:
                    continue
                for t in range(8):
                    e = p * kp + 8 * v + t
                    pr = np.float32(w[e]) * np.float32(x[e])
                    if t % 2 == 0:
                        a0 = np.float32(a0 + pr)
                    else:
                        a1 = np.float32(a1 + pr)
            lanes.append(np.float32(a0 + a1))
        a = np.array(lanes, np.float32)
        for o in (16, 8, 4, 2, 1):
            a = (a + a[np.arange(32) ^ o]).astype(np.float32)
        parts.append(a[0])
    d = parts[0]
    for q in parts[1:]:
        d = np.float32(d + q)
    return d


@pytest.mark.parametrize("K", [128, 384, 512, 1408, 2048, 10944])
def test_dot_rows_is_the_specified_order(K):
    """The vectorised emulation equals the order spelled out scalar by scalar, and stays within
    FP32 accumulation error of the exact dot product."""
    rng = np.random.default_rng(K)
    W = D.bf16(rng.standard_normal((3, K)).astype(np.float32) * 0.02)
    x = D.bf16(rng.standard_normal(K).astype(np.float32))
    got = D.dot_rows(W, x)
    want = np.array([_scalar_row_dot(W[i], x) for i in range(3)], np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    exact = W.astype(np.float64) @ x.astype(np.float64)
    assert np.all(np.abs(got - exact) <= 1e-5 * np.abs(W).sum(1) * np.abs(x).max())


def test_gemv_partition():
    assert D.gemv_parts(2048) == (8, 256, 1)
    assert D.gemv_parts(1408) == (8, 176, 1)
    assert D.gemv_parts(1024) == (4, 256, 1)
    assert D.gemv_parts(512) == (2, 256, 1)
    assert D.gemv_parts(384) == (2, 192, 1)
    assert D.gemv_parts(128) == (1, 128, 1)
    assert D.gemv_parts(10944) == (8, 1368, 6)


def test_block_and_lane_sums():
    rng = np.random.default_rng(6)
    v = rng.standard_normal(2048).astype(np.float32)
    acc = np.zeros(256, np.float32)
    for i in range(8):
        acc = (acc + v[i * 256:(i + 1) * 256]).astype(np.float32)
    w = D.butterfly(acc.reshape(8, 32))
    tot = w[0]
    for k in range(1, 8):
        tot = np.float32(tot + w[k])
    assert D.block_sum(v, vec=1) == tot
    assert abs(float(D.lane_sum(v[:70])) - float(v[:70].astype(np.float64).sum())) < 1e-5
    assert D.seq_sum(v[:5]) == np.float32(np.float32(np.float32(np.float32(v[0] + v[1]) + v[2]) + v[3]) + v[4])


# ---- the C restatement of the hot loops (oracle/detdot.c) equals the numpy specification

def _c_lib():
    from oracle import detmath as D
    L = D._od()
    if L is None:
        pytest.skip("oracle/libdetdot.so is not built (make -C oracle)")
    return D, L


@pytest.mark.parametrize("K", [64, 96, 128, 256, 512, 1024, 1408, 2048, 10944])
def test_c_dot_rows_equals_numpy(K):
    D, _ = _c_lib()
    rng = np.random.default_rng(K)
    W = D.bf16((rng.standard_normal((29, K)) * 0.02).astype(np.float32))
    x = D.bf16(rng.standard_normal(K).astype(np.float32))
    want = D.dot_rows_np(W, x).view(np.uint32)
    assert np.array_equal(D.dot_rows(W, x).view(np.uint32), want)
    assert np.array_equal(D.dot_rows(D.bf16_bits(W), x).view(np.uint32), want)


def test_c_exp_log_equal_numpy():
    D, L = _c_lib()
    rng = np.random.default_rng(5)
    xs = np.concatenate([(rng.standard_normal(4000) * 30).astype(np.float32),
                         np.array([-87, -87.5, 88, 88.1, 0, -0.0, 1e-40, 1e-38, np.inf, -np.inf], np.float32)])
    got = np.array([L.od_det_exp(float(v)) for v in xs], np.float32)
    assert np.array_equal(got.view(np.uint32), D.det_exp(xs).view(np.uint32))
    ys = np.concatenate([np.abs(xs), np.array([1e-42, 1e-39, 3.4e38], np.float32)])
    got = np.array([L.od_det_log(float(v)) for v in ys], np.float32)
    assert np.array_equal(got.view(np.uint32), D.det_log(ys).view(np.uint32))


@pytest.mark.parametrize("nh,dc,dr,s,pos,split", [(16, 512, 64, 1100, 1050, 128), (4, 64, 16, 300, 250, 24),
                                                  (16, 512, 64, 200, 63, 32)])
def test_c_mla_attend_equals_numpy(nh, dc, dr, s, pos, split):
    D, _ = _c_lib()
    from oracle import numpy_ref as R
    rng = np.random.default_rng(pos)
    bf = lambda *sh: D.bf16(rng.standard_normal(sh).astype(np.float32))  # noqa: E731
    args = (bf(nh, dc), bf(nh, dr), bf(s, dc), bf(s, dr), pos, 0.11)
    got = R.mla_attend(*args, split=split)
    saved, D._OD_LIB = D._OD_LIB, False
    try:
        want = R.mla_attend(*args, split=split)
    finally:
        D._OD_LIB = saved
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ---- FP8 (E4M3) experts ----------------------------------------------------------------------


def test_e4m3_table_matches_torch():
    """The oracle's E4M3 decoding (from the format's definition) equals torch.float8_e4m3fn on all
    256 codes (NaN codes 0x7F and 0xFF included)."""
    from oracle import numpy_ref as R
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    want = codes.view(torch.float8_e4m3fn).float().numpy()
    got = R.e4m3(np.arange(256))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok].view(np.uint32), want[ok].view(np.uint32))
    assert R.e4m3(np.array([0x7E]))[0] == 448.0 and R.e4m3(np.array([0x01]))[0] == 2.0 ** -9


def test_quantize_e4m3_scales_and_codes():
    """Per-tensor scales amax / 448 (gate and up rows of the interleaved W13 apart); every code is a
    finite E4M3 value; the largest weight of a tensor maps to +-448 and decoding times the scale
    stays within half an E4M3 step of each weight; an all-zero tensor gets scale 1."""
    from fleet.pack_weights import fp8_experts, quantize_e4m3, regroup_w2
    from oracle import numpy_ref as R
    g = torch.Generator().manual_seed(5)
    W13 = (0.02 * torch.randn(3, 2 * 64, 96, generator=g)).to(torch.bfloat16)
    W13[2] = 0
    q, s = quantize_e4m3(W13, 2)
    assert q.dtype == torch.uint8 and s.shape == (3, 2)
    w = W13.float().numpy()
    for e in range(2):
        for p in range(2):
            rows = w[e, p::2]
            assert np.float32(s[e, p]) == np.float32(np.abs(rows).max() / np.float32(448.0))
            dec = R.e4m3(q[e, p::2].numpy())
            assert np.isfinite(dec).all() and np.abs(dec).max() == 448.0
            err = np.abs(dec * s[e, p].item() - rows)
            assert (err <= np.abs(rows) * 2.0 ** -4 + 2.0 ** -10 * s[e, p].item()).all()
    assert s[2].tolist() == [1.0, 1.0] and int(q[2].sum()) == 0
    W2 = (0.02 * torch.randn(3, 96, 64, generator=g)).to(torch.bfloat16)
    W13q, s13, W2Fq, s2 = fp8_experts(W13, W2)
    W2q, s2b = quantize_e4m3(W2, 1)
    assert torch.equal(W13q, q) and torch.equal(s13, s) and torch.equal(s2, s2b.reshape(-1))
    assert torch.equal(W2Fq, regroup_w2(W2q))


def test_linear_fp8_is_exact_products_in_row_order():
    """linear_fp8 = bf16(scale * dot_rows(e4m3(q), f16(x))): each product is exact (4 x 11
    significant bits), so the dot is the row-dot order over exact products; close to the FP64 dot."""
    from oracle import numpy_ref as R
    rng = np.random.default_rng(9)
    q = rng.integers(0, 256, size=(16, 1408), dtype=np.uint8)
    q[(q & 0x7F) == 0x7F] = 0x00                                   # no NaN codes
    x = R.bf16(rng.standard_normal(1408).astype(np.float32))
    y = R.linear_fp8(x, q, np.float32(0.01))
    xd = R.f16(x).astype(np.float64)
    ref = 0.01 * (R.e4m3(q).astype(np.float64) @ xd)
    assert np.allclose(y, ref, rtol=2e-2, atol=1e-2 * np.abs(ref).max())
    assert np.array_equal(y, R.bf16((np.float32(0.01) * D.dot_rows(R.e4m3(q), R.f16(x))).astype(np.float32)))


def test_f16_activation_rounding():
    """The FP8 path's activation operand: exact for BF16 values of magnitude in [2^-14, 65504],
    nearest-even below, saturated at +-65504 above (the kernel's cvt.rn.satfinite)."""
    from oracle import numpy_ref as R
    x = np.array([1.0, -3.5, 2.0 ** -14, 65504.0, 65536.0, -1e30, 2.0 ** -20 * 1.5, 2.0 ** -26, np.nan], np.float32)
    y = R.f16(x)
    assert y[:4].tolist() == [1.0, -3.5, 2.0 ** -14, 65504.0]
    assert y[4] == 65504.0 and y[5] == -65504.0
    assert y[6] == np.float32(np.float16(2.0 ** -20 * 1.5)) and y[7] == 0.0 and np.isnan(y[8])
    b = R.bf16(np.random.default_rng(3).standard_normal(4096).astype(np.float32) * 100)
    ok = (np.abs(b) >= 2.0 ** -14) & (np.abs(b) <= 65504)
    assert np.array_equal(R.f16(b)[ok], b[ok])
