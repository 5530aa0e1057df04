"""Parity of every sm_100a task kernel with the CPU oracle, through the C ABI.

Each test builds a small operator chain with the library (fleet/mk.py -> include/fleet_mk.h),
runs it in the persistent kernel on cuda:0 and compares with oracle/numpy_ref.py on the same
seeded inputs. The bar is BIT-EXACT equality of every BF16/FP32/int output: the kernels and the
oracle make the same arithmetic choices (exact dot products rounded once, det_exp/det_log), so
any difference is a bug, not rounding noise. Shapes are DeepSeek-V2-Lite's.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import DeviceWeights, assert_bits_equal, bits, np32, rnd_bf16
from oracle import detmath as D
from oracle import numpy_ref as R
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def mk():
    from fleet import mk as _mk
    _mk.lib()
    return _mk


@pytest.fixture(scope="module")
def B():
    from fleet import build_graph
    return build_graph


def run_ops(mk, ops, iters=1, step=0, num_ctas=0, timeout=5.0):
    k = mk.MegaKernel(0, num_ctas=num_ctas, wait_timeout_s=timeout)
    for op in ops:
        k.add(op)
    k.finalize()
    k.launch(iters, step)
    st = k.status()
    torch.cuda.synchronize()
    assert st["error"] == 0, st
    return k


def gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


# ---------------------------------------------------------------------------------------------


def test_device_detmath_bit_exact(mk):
    rng = np.random.default_rng(0)
    specials = [0.0, -0.0, np.inf, -np.inf, np.nan, -87.0, 88.0, 88.5, -87.5, 1e-40, -1e-40]
    x = np.concatenate([rng.uniform(-90, 90, 1 << 20), rng.uniform(-1, 1, 1 << 18), specials]).astype(np.float32)
    xt = torch.from_numpy(x).to(DEV)
    out = torch.empty_like(xt)

    def same(a, b):
        a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
        return np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(
            a[~np.isnan(a)].view(np.uint32), b[~np.isnan(b)].view(np.uint32))

    mk.selftest_math(0, xt, out)
    assert same(out.cpu().numpy(), D.det_exp(x))
    pos = np.concatenate([np.exp(rng.uniform(-85, 85, 1 << 19)), rng.uniform(0.5, 40, 1 << 18),
                          [1.0, 2.0, 1e-40, 3e-45, 0.0, np.inf]]).astype(np.float32)
    pt = torch.from_numpy(pos).to(DEV)
    out = torch.empty_like(pt)
    mk.selftest_math(1, pt, out)
    assert same(out.cpu().numpy(), D.det_log(pos))
    out = torch.empty_like(xt)
    mk.selftest_math(2, xt, out)
    assert same(out.cpu().numpy(), D.silu(x))
    x64 = np.concatenate([rng.standard_normal(1 << 18) * np.exp(rng.uniform(-40, 40, 1 << 18)),
                          [1.0 + 2 ** -8 + 2 ** -40, 1.0 + 2 ** -8, 2.0 ** -130, -3 * 2.0 ** -134, 3.5e38]])
    x64t = torch.from_numpy(x64).to(DEV)
    o16 = torch.empty(x64.size, dtype=torch.int16, device=DEV)
    mk.selftest_math(3, x64t, o16)
    assert np.array_equal(o16.cpu().numpy().view(np.uint16), D.bf16_bits(D.bf16_from_f64(x64)))
    o16 = torch.empty(x.size, dtype=torch.int16, device=DEV)
    fin = torch.from_numpy(np.nan_to_num(x, nan=1.0)).to(DEV)
    mk.selftest_math(4, fin, o16)
    assert np.array_equal(o16.cpu().numpy().view(np.uint16), D.bf16_bits(D.bf16(np.nan_to_num(x, nan=1.0))))


GEMV_CASES = [
    (3648, 2048, "norm", 0),        # qkva with the input RMSNorm
    (2048, 2048, "res", 0),         # o_proj + residual
    (1000, 1408, "plain", 0),       # K of the expert down projection, odd N
    (512, 512, "plain", 0),
    (300, 128, "plain", 0),
    (2048, 10944, "res", 0),        # layer 0's down projection (K split over the warps)
    (102400, 2048, "norm_argmax", 0),
    (3648, 2048, "norm", 7),        # a 7-CTA schedule: several tasks per CTA
]


@pytest.mark.parametrize("N,K,kind,ctas", GEMV_CASES)
def test_gemv(mk, B, N, K, kind, ctas):
    g = gen(N + K)
    W = rnd_bf16(g, N, K, std=0.02)
    x = rnd_bf16(g, K)
    w_norm = (1.0 + 0.5 * torch.randn(K, generator=g, device=DEV)).to(torch.bfloat16)
    res = rnd_bf16(g, N)
    out = torch.zeros(N, dtype=torch.bfloat16, device=DEV)
    hout = torch.zeros(K, dtype=torch.bfloat16, device=DEV)
    tokens = torch.zeros(1, 8, dtype=torch.int64, device=DEV)
    norm, resid, argmax = "norm" in kind, kind == "res", "argmax" in kind
    op = B.linear_gemv_layer(mk, None, input=x, weight=W, output=out, w_norm=w_norm if norm else None,
                             residual=res if resid else None, h_out=hout if norm else None,
                             tokens_out=tokens if argmax else None, norm=norm, residual_add=resid, argmax=argmax)
    run_ops(mk, [op], step=2, num_ctas=ctas)
    xin = R.rmsnorm(np32(x), np32(w_norm)) if norm else np32(x)
    want = R.linear_residual(xin, np32(W), np32(res)) if resid else R.linear(xin, np32(W))
    assert_bits_equal(out, want, f"gemv {N}x{K} {kind}")
    if norm:
        assert_bits_equal(hout, xin, "normalised row")
    if argmax:
        assert int(tokens[0, 4]) == int(np.argmax(want))


def test_argmax_ties_to_lower_index(mk, B):
    N, K = 4096, 2048
    g = gen(11)
    W = rnd_bf16(g, N, K, std=0.02)
    x = rnd_bf16(g, K)
    w_norm = torch.ones(K, dtype=torch.bfloat16, device=DEV)
    y = R.linear(R.rmsnorm(np32(x), np32(w_norm)), np32(W))
    top = int(np.argmax(y))
    lo = 5 if top > 5 else top + 100
    W[lo] = W[top]                                  # a bit-identical logit in another task's rows
    W[N - 1] = W[top]
    out = torch.zeros(N, dtype=torch.bfloat16, device=DEV)
    tokens = torch.zeros(1, 8, dtype=torch.int64, device=DEV)
    op = B.linear_gemv_layer(mk, None, input=x, weight=W, output=out, w_norm=w_norm, tokens_out=tokens, norm=True,
                             argmax=True)
    run_ops(mk, [op], step=0)                       # position 1: the token goes to tokens[2]
    assert int(tokens[0, 2]) == min(lo, top)


@pytest.mark.parametrize("pos", [1024, 1023, 700, 64])
def test_mla_prep_attend_merge(mk, B, pos):
    nh, d_n, d_r, d_c, d_v, s_max, split, hg = 16, 128, 64, 512, 128, 1056, 128, 1
    n_splits = -(-s_max // split)
    g = gen(pos)
    qkva = rnd_bf16(g, nh * (d_n + d_r) + d_c + d_r)
    w_kv = (1.0 + 0.5 * torch.randn(d_c, generator=g, device=DEV)).to(torch.bfloat16)
    W_ukT = rnd_bf16(g, nh, d_c, d_n, std=0.05)
    W_uv = rnd_bf16(g, nh, d_v, d_c, std=0.05)
    from fleet.capture import rope_tables, softmax_scale
    cos, sin = rope_tables(d_r, s_max, device=DEV)
    c_kv = rnd_bf16(g, s_max, d_c)
    k_pe = rnd_bf16(g, s_max, d_r)
    c_kv[pos:] = 0
    k_pe[pos:] = 0
    c0, k0 = np32(c_kv), np32(k_pe)
    qln = torch.zeros(nh, d_c, dtype=torch.bfloat16, device=DEV)
    qpe = torch.zeros(nh, d_r, dtype=torch.bfloat16, device=DEV)
    from fleet.graph_plan import partials_row
    partials = torch.full((n_splits, nh, partials_row(d_c)), 7.0, dtype=torch.float32, device=DEV)
    attn = torch.zeros(nh * d_v, dtype=torch.bfloat16, device=DEV)
    scale = softmax_scale(d_n, d_r)
    ops = [B.mla_prep_layer(mk, None, qkva, w_kv, W_ukT, cos, sin, c_kv, k_pe, qln, qpe),
           B.mla_attend_layer(mk, None, qln, qpe, c_kv, k_pe, partials, scale, split, n_splits, hg),
           B.mla_merge_uv_layer(mk, None, partials, W_uv, attn, split, n_splits)]
    run_ops(mk, ops, step=pos - 1)
    W_uk = np32(W_ukT).transpose(0, 2, 1)
    c_row, k_row, ql, q_pe = R.mla_prep(np32(qkva), np32(w_kv), W_uk, np32(cos)[pos], np32(sin)[pos])
    assert_bits_equal(c_kv[pos], c_row, "c_kv row")
    assert_bits_equal(k_pe[pos], k_row, "k_pe row")
    assert_bits_equal(qln, ql, "ql_nope")
    assert_bits_equal(qpe, q_pe, "q_pe")
    assert np.array_equal(np32(c_kv)[:pos], c0[:pos]) and not np32(c_kv)[pos + 1:].any()   # other rows untouched
    c0[pos], k0[pos] = c_row, k_row
    want = R.mla_attend(ql, q_pe, c0, k0, pos, scale, split=split, n_splits=n_splits)
    got = partials.cpu().numpy()
    assert np.array_equal(got[:, :, :d_c + 1].view(np.uint32), want.view(np.uint32)), "partials differ"
    assert np.all(got[:, :, d_c + 1:] == 7.0)                                       # padding untouched
    assert_bits_equal(attn, R.mla_merge_uv(want, np32(W_uv), pos, split=split), "attn")


# Config C2, the MLA decode-attention sweep: contexts 1K..32K with N(0,1) BF16 q and latent KV
# (seed 3). At 1K the split factors 8 / 16 / 32 are splits of 128 / 64 / 32 rows; longer contexts
# keep 128-row splits (a split's rows must fit the weight ring), 32 to 256 of them per head, which
# the merge adds in order. A head group > 1 (the plan's choice at long context) runs several heads
# of one split in one task over the same ring stages: the same partials, bit for bit.
@pytest.mark.parametrize("ctx,split,hg", [(1024, 128, 1), (1024, 64, 1), (1024, 32, 1), (4096, 128, 1),
                                          (4096, 128, 2), (8192, 128, 4), (16384, 128, 1), (16384, 128, 8),
                                          (32768, 128, 1)])
def test_mla_attend_merge_long_context(mk, B, ctx, split, hg):
    nh, d_r, d_c, d_v = 16, 64, 512, 128
    s_max = ctx
    n_splits = -(-s_max // split)
    pos = ctx - 1
    g = gen(3)
    ql = rnd_bf16(g, nh, d_c)
    qp = rnd_bf16(g, nh, d_r)
    c_kv = rnd_bf16(g, s_max, d_c)
    k_pe = rnd_bf16(g, s_max, d_r)
    W_uv = rnd_bf16(g, nh, d_v, d_c, std=0.05)
    from fleet.capture import softmax_scale
    from fleet.graph_plan import partials_row
    partials = torch.zeros((n_splits, nh, partials_row(d_c)), dtype=torch.float32, device=DEV)
    attn = torch.zeros(nh * d_v, dtype=torch.bfloat16, device=DEV)
    scale = softmax_scale(128, d_r)
    ops = [B.mla_attend_layer(mk, None, ql, qp, c_kv, k_pe, partials, scale, split, n_splits, hg),
           B.mla_merge_uv_layer(mk, None, partials, W_uv, attn, split, n_splits)]
    run_ops(mk, ops, step=pos - 1)
    want = R.mla_attend(np32(ql), np32(qp), np32(c_kv), np32(k_pe), pos, scale, split=split, n_splits=n_splits)
    got = partials.cpu().numpy()
    assert np.array_equal(got[:, :, :d_c + 1].view(np.uint32), want.view(np.uint32)), "partials differ"
    assert_bits_equal(attn, R.mla_merge_uv(want, np32(W_uv), pos, split=split), "attn")


# The tensor-core form (MK_F_TC): all 16 heads of a split in one task, mma.sync with FP32
# accumulation in the tensor cores' order. Config 2's sweep: contexts 1K..32K, 8/16/32 splits (a
# split of ctx / n rows, processed in chunks of 96 rows with an online softmax), plus positions
# whose own row is alone in its chunk or split. Within the north-star tolerance of the oracle's
# specified-order result: partials and attn max-abs error <= 2e-2 of the largest value, lse
# within 1e-3, cosine >= 0.9999.
def _close(got, want, what, rel=2e-2, cos=0.9999):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    err = np.abs(got - want).max()
    scale = np.abs(want).max()
    c = float(got @ want / (np.linalg.norm(got) * np.linalg.norm(want) + 1e-30))
    assert err <= rel * scale and c >= cos, f"{what}: max err {err:.3g} (scale {scale:.3g}), cosine {c:.6f}"


@pytest.mark.parametrize("ctx,n_splits,pos,parts", [
    (1024, 8, None, 1), (1024, 16, None, 1), (1024, 32, None, 1), (4096, 8, None, 1), (4096, 16, None, 1),
    (4096, 32, None, 1), (16384, 8, None, 1), (16384, 32, None, 1), (32768, 8, None, 1), (32768, 16, None, 1),
    (32768, 32, None, 1), (1056, 11, 1055 - 96, 1), (1056, 11, 96 * 3, 1), (1056, 11, 0, 1), (1056, 11, 5, 1),
    (1056, 11, 1024, 1), (1024, 16, None, 2), (1024, 16, None, 4), (4096, 16, None, 8), (1056, 11, 5, 4),
    (1056, 33, 1024, 4)])
def test_mla_attend_tc_matches_oracle(mk, B, ctx, n_splits, pos, parts):
    nh, d_r, d_c, d_v = 16, 64, 512, 128
    s_max = ctx
    split = -(-ctx // n_splits)
    pos = ctx - 1 if pos is None else pos
    g = gen(3)
    ql = rnd_bf16(g, nh, d_c)
    qp = rnd_bf16(g, nh, d_r)
    c_kv = rnd_bf16(g, s_max, d_c)
    k_pe = rnd_bf16(g, s_max, d_r)
    W_uv = rnd_bf16(g, nh, d_v, d_c, std=0.05)
    from fleet.capture import softmax_scale
    from fleet.graph_plan import partials_row
    partials = torch.zeros((n_splits, nh, partials_row(d_c)), dtype=torch.float32, device=DEV)
    attn = torch.zeros(nh * d_v, dtype=torch.bfloat16, device=DEV)
    scale = softmax_scale(128, d_r)
    ops = [B.mla_attend_layer(mk, None, ql, qp, c_kv, k_pe, partials, scale, split, n_splits, nh, tc=True,
                              col_parts=parts),
           B.mla_merge_uv_layer(mk, None, partials, W_uv, attn, split, n_splits)]
    run_ops(mk, ops, step=pos - 1)
    want = R.mla_attend(np32(ql), np32(qp), np32(c_kv), np32(k_pe), pos, scale, split=split, n_splits=n_splits)
    got = partials.cpu().numpy()
    live = -(-(pos + 1) // split)
    assert np.all(np.isneginf(got[live:, :, d_c])) and not np.any(got[live:, :, :d_c]), "dead splits"
    _close(got[:live, :, :d_c], want[:live, :, :d_c], "partials o")
    assert np.abs(got[:live, :, d_c] - want[:live, :, d_c]).max() <= 1e-3, "partials lse"
    _close(np32(attn), R.mla_merge_uv(want, np32(W_uv), pos, split=split), "attn")


def _router_inputs(g, E=64, H=2048):
    x = rnd_bf16(g, H)
    w_norm = (1.0 + 0.5 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    W_gate = rnd_bf16(g, E, H, std=0.02)
    return x, w_norm, W_gate


def _router_bufs(E=64, NS=8, H=2048, L=26):
    z = dict(device=DEV)
    return dict(h=torch.zeros(H, dtype=torch.bfloat16, **z), topk_w=torch.zeros(NS, dtype=torch.float32, **z),
                routing=torch.zeros(E + 2, dtype=torch.int32, **z), mask=torch.zeros(E + 3, dtype=torch.int32, **z),
                logits=torch.zeros(E, dtype=torch.float32, **z),
                route_log=torch.full((32, L, NS), -9, dtype=torch.int32, **z))


@pytest.mark.parametrize("tie", [False, True])
def test_router(mk, B, tie):
    g = gen(21 + tie)
    x, w_norm, W_gate = _router_inputs(g)
    if tie:
        h = R.rmsnorm(np32(x), np32(w_norm))
        top = int(np.argmax(R.linear(h, np32(W_gate))))
        other = (top + 17) % 64
        W_gate[other] = W_gate[top]
    b = _router_bufs()
    op = B.moe_router_layer(mk, None, x, w_norm, W_gate, b["h"], b["topk_w"], b["routing"], b["mask"], b["logits"],
                            b["route_log"], layer_index=3, topk=6, n_experts=64, n_forced=2, scaling=1.0, eps=1e-6)
    run_ops(mk, [op])
    h, logits, topk_w, routing, mask = R.moe_router_norm(np32(x), np32(w_norm), np32(W_gate))
    assert_bits_equal(b["h"], h, "router h")
    assert np.array_equal(b["logits"].cpu().numpy().view(np.uint32), logits.view(np.uint32))
    assert np.array_equal(b["topk_w"].cpu().numpy().view(np.uint32), topk_w.view(np.uint32))
    assert np.array_equal(b["routing"].cpu().numpy(), routing)
    assert np.array_equal(b["mask"].cpu().numpy(), mask)
    assert b["route_log"][0, 3].tolist() == mask[:8].tolist()
    if tie:
        lo, hi = sorted((top, other))
        assert mask[0] == lo and mask[1] == hi


def test_router_bias_skewed(mk, B):
    """Injected routing (config 3): a Zipf-shaped logit bias moves the choice as the oracle says."""
    g = gen(31)
    x, w_norm, W_gate = _router_inputs(g)
    ranks = np.random.default_rng(4).permutation(64) + 1
    bias = (3.0 * (1.0 / ranks ** 1.2)).astype(np.float32)
    bias_t = torch.from_numpy(bias).to(DEV)
    b = _router_bufs()
    op = B.moe_router_layer(mk, None, x, w_norm, W_gate, b["h"], b["topk_w"], b["routing"], b["mask"], b["logits"],
                            b["route_log"], layer_index=0, topk=6, n_experts=64, n_forced=2, scaling=1.0, eps=1e-6,
                            bias=bias_t)
    run_ops(mk, [op])
    _, logits, topk_w, _, mask = R.moe_router_norm(np32(x), np32(w_norm), np32(W_gate), logit_bias=bias)
    assert np.array_equal(b["mask"].cpu().numpy(), mask)
    assert np.array_equal(b["topk_w"].cpu().numpy().view(np.uint32), topk_w.view(np.uint32))


def test_moe_block(mk, B):
    """router -> w13 (+SwiGLU) -> w2 (+ combine into x_res), real shapes, 8 slots of 66 experts."""
    from fleet.pack_weights import REAL_DIMS as d
    g = gen(41)
    x, w_norm, W_gate = _router_inputs(g)
    W13 = rnd_bf16(g, d.E_TOTAL, 2 * d.I_MOE, d.H, std=0.02)
    W2 = rnd_bf16(g, d.E_TOTAL, d.H, d.I_MOE, std=0.02)
    b = _router_bufs()
    mid = torch.zeros(8, 2 * d.I_MOE, dtype=torch.bfloat16, device=DEV)
    act8 = torch.zeros(8, d.I_MOE, dtype=torch.bfloat16, device=DEV)
    out8 = torch.zeros(8, d.H, dtype=torch.bfloat16, device=DEV)
    x_res = x.clone()
    ops = [B.moe_router_layer(mk, None, x_res, w_norm, W_gate, b["h"], b["topk_w"], b["routing"], b["mask"],
                              b["logits"], b["route_log"], layer_index=0, topk=6, n_experts=64, n_forced=2,
                              scaling=1.0, eps=1e-6),
           B.gateup_layer(mk, None, b["h"], W13, act8, inter=d.I_MOE, groups=8, expert=True, norm=False,
                          mask=b["mask"], mid=mid),
           B.moe_w2_combine_layer(mk, None, act8, W2, b["mask"], b["topk_w"], x_res, x_res, out8)]
    run_ops(mk, ops)
    dw = DeviceWeights({"W13": W13, "W2": W2})
    h, logits, topk_w, routing, mask = R.moe_router_norm(np32(x), np32(w_norm), np32(W_gate))
    assert np.array_equal(b["mask"].cpu().numpy(), mask)
    want_mid = np.stack([R.linear(h, OracleModel.gate_up(dw.get_expert("W13", int(e)))) for e in mask[:8]])
    assert_bits_equal(mid, want_mid, "mid")
    want_act = np.stack([R.swiglu_act(m, d.I_MOE) for m in want_mid])
    assert_bits_equal(act8, want_act, "act")
    want_out8 = np.stack([R.linear(a, dw.get_expert("W2", int(e))) for a, e in zip(want_act, mask[:8])])
    assert_bits_equal(out8, want_out8, "out8")
    assert_bits_equal(x_res, R.moe_combine(want_out8, topk_w, np32(x)), "combined x_res")


@pytest.mark.parametrize("H,I,E,topk,nf,tags,beside", [(2048, 1408, 64, 6, 2, True, False),
                                                      (2048, 1408, 64, 6, 2, True, True),
                                                      (2048, 1408, 64, 6, 2, False, False),
                                                      (64, 96, 8, 2, 2, True, False),
                                                      (128, 256, 12, 3, 1, False, True),
                                                      (256, 1024, 8, 2, 1, True, False)])
def test_moe_units_block(mk, B, H, I, E, topk, nf, tags, beside):
    """The expert units: router -> the units of every slot (each task normalises x_res itself, runs
    its share of the shared slots' units with their fixed experts, then its share of the routed
    slots' units with the router's experts) -> the combine into x_res; out8, the
    activations and x_res equal the oracle's staged arithmetic (w13 + SwiGLU, w2 row dots in the
    row engine's order, moe_combine) bit for bit. The shapes cover 22 lanes in 8 parts (the model),
    12 lanes in one part (classes of one and two lanes), 32 lanes in one part (four-lane classes)
    and 32 lanes in four parts. tags: the router hands its logits to its task 0 and the slots'
    experts to the units as tagged words (the decode graph's form), else through its arrival
    counter and completion event. beside: the units take one task per CTA and their last tasks, on
    the router's CTAs, run routed units only (MK_I_MU_FTASKS, the decode graph's form)."""
    from fleet.pack_weights import unit_parts
    g = gen(43 + H)
    ns = topk + nf
    x = rnd_bf16(g, H)
    w_norm = (1.0 + 0.5 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    W_gate = rnd_bf16(g, E, H, std=0.05)
    W13 = rnd_bf16(g, E + nf, 2 * I, H, std=0.02)
    W2 = rnd_bf16(g, E + nf, H, I, std=0.02)
    W2F = B.regrouped_w2(W2)
    b = _router_bufs(E=E, NS=ns, H=H, L=1)
    sums = torch.full((ns, unit_parts(I), 8, H), float("nan"), dtype=torch.float32, device=DEV)
    act8 = torch.zeros(ns, I, dtype=torch.bfloat16, device=DEV)
    out8 = torch.zeros(ns, H, dtype=torch.bfloat16, device=DEV)
    x_res = x.clone()
    tag = {}
    if tags:
        tag = dict(logit_tag=torch.zeros(E, dtype=torch.int64, device=DEV),
                   mask_tag=torch.zeros(ns, dtype=torch.int64, device=DEV))
    ops = [B.moe_router_layer(mk, None, x_res, w_norm, W_gate, b["h"], b["topk_w"], b["routing"], b["mask"],
                              b["logits"], b["route_log"], layer_index=0, topk=topk, n_experts=E, n_forced=nf,
                              scaling=1.0, eps=1e-6, **tag),
           B.moe_units_layer(mk, None, x_res, W13, W2F, sums, slot0=0, nslots=ns, inter=I, w_norm=w_norm,
                             mask=b["mask"], act=act8, norm=True, fixed0=topk, static_experts=E,
                             mask_tag=tag.get("mask_tag")),
           B.moe_combine_layer(mk, None, sums, b["topk_w"], x_res, x_res, inter=I, out8=out8)]
    if beside:
        n_cta = torch.cuda.get_device_properties(0).multi_processor_count
        n_rt = 8 if E % 8 == 0 else 4
        ops[0].ntasks = n_rt
        ops[1].ntasks = n_cta
        ops[1].ip[mk.P["mu_i"]["FTASKS"]] = n_cta - n_rt
    run_ops(mk, ops)
    dw = DeviceWeights({"W13": W13, "W2": W2})
    h, logits, topk_w, routing, mask = R.moe_router_norm(np32(x), np32(w_norm), np32(W_gate), topk=topk,
                                                         n_experts=E, forced=tuple(range(E, E + nf)))
    assert np.array_equal(b["mask"].cpu().numpy()[:ns], mask[:ns])
    want_act = np.stack([R.swiglu_act(R.linear(h, OracleModel.gate_up(dw.get_expert("W13", int(e)))), I)
                         for e in mask[:ns]])
    assert_bits_equal(act8, want_act, "act")
    want_out8 = np.stack([R.linear(a, dw.get_expert("W2", int(e))) for a, e in zip(want_act, mask[:ns])])
    assert_bits_equal(out8, want_out8, "out8")
    assert_bits_equal(x_res, R.moe_combine(want_out8, topk_w, np32(x)), "combined x_res")


@pytest.mark.parametrize("H,I,E,topk,nf,sat", [(2048, 1408, 64, 6, 2, False), (2048, 1408, 64, 6, 2, True),
                                              (64, 96, 8, 2, 2, False), (256, 1024, 8, 2, 1, False)])
def test_moe_units_fp8_block(mk, B, H, I, E, topk, nf, sat):
    """Weight-only FP8 experts (E4M3 codes, one scale per gate, up and down tensor of each expert):
    router -> FP8 expert units -> combine with the down scales; the activations, out8 and x_res
    equal the oracle's FP8 form (moe_experts_fp8: FP16-rounded activations, exact products, the
    row-dot order, the scale on each row's total, BF16) bit for bit. The codes include subnormal
    E4M3 values (exponent field 0). sat: one normalised activation far beyond the FP16 range
    (saturated at 65504 for the products, as the oracle's f16 does)."""
    from fleet.pack_weights import fp8_experts, quantize_e4m3, unit_parts
    g = gen(47 + H)
    ns = topk + nf
    x = rnd_bf16(g, H)
    w_norm = (1.0 + 0.5 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    if sat:
        w_norm[7] = 65536.0                 # h[7] ~ 65536 x[7] / rms(x), rms(x) ~ 1: >> 65504
        x[7] = 4.0
    W_gate = rnd_bf16(g, E, H, std=0.05)
    W13 = rnd_bf16(g, E + nf, 2 * I, H, std=0.02)
    W2 = rnd_bf16(g, E + nf, H, I, std=0.02)
    W13q, s13, W2Fq, s2 = fp8_experts(W13, W2)
    W2q, _ = quantize_e4m3(W2, 1)
    sub = ((W13q & 0x78) == 0) & ((W13q & 0x07) != 0)
    assert bool(sub.any()) or H * I < 2 ** 16, "no subnormal codes"
    b = _router_bufs(E=E, NS=ns, H=H, L=1)
    sums = torch.full((ns, unit_parts(I), 8, H), float("nan"), dtype=torch.float32, device=DEV)
    act8 = torch.zeros(ns, I, dtype=torch.bfloat16, device=DEV)
    out8 = torch.zeros(ns, H, dtype=torch.bfloat16, device=DEV)
    x_res = x.clone()
    tag = dict(logit_tag=torch.zeros(E, dtype=torch.int64, device=DEV),
               mask_tag=torch.zeros(ns, dtype=torch.int64, device=DEV))
    ops = [B.moe_router_layer(mk, None, x_res, w_norm, W_gate, b["h"], b["topk_w"], b["routing"], b["mask"],
                              b["logits"], b["route_log"], layer_index=0, topk=topk, n_experts=E, n_forced=nf,
                              scaling=1.0, eps=1e-6, **tag),
           B.moe_units_layer(mk, None, x_res, W13q, W2Fq, sums, slot0=0, nslots=ns, inter=I, w_norm=w_norm,
                             mask=b["mask"], act=act8, norm=True, fixed0=topk, static_experts=E,
                             mask_tag=tag["mask_tag"], scale13=s13),
           B.moe_combine_layer(mk, None, sums, b["topk_w"], x_res, x_res, inter=I, out8=out8, mask=b["mask"],
                               scale2=s2)]
    run_ops(mk, ops)
    h, logits, topk_w, routing, mask = R.moe_router_norm(np32(x), np32(w_norm), np32(W_gate), topk=topk,
                                                         n_experts=E, forced=tuple(range(E, E + nf)))
    assert not sat or abs(h[7]) > 65504
    assert np.array_equal(b["mask"].cpu().numpy()[:ns], mask[:ns])
    want_act, want_out8 = R.moe_experts_fp8(h, W13q.cpu().numpy(), s13.cpu().numpy(), W2q.cpu().numpy(),
                                            s2.cpu().numpy(), mask, n_slots=ns)
    assert_bits_equal(act8, want_act, "act")
    assert_bits_equal(out8, want_out8, "out8")
    assert_bits_equal(x_res, R.moe_combine(want_out8, topk_w, np32(x)), "combined x_res")


def test_dense_mlp(mk, B):
    """Layer 0: norm2 + gate/up (+SwiGLU) over I 10,944, then the K-split down projection."""
    from fleet.pack_weights import REAL_DIMS as d
    g = gen(51)
    x = rnd_bf16(g, d.H)
    w_norm = (1.0 + 0.5 * torch.randn(d.H, generator=g, device=DEV)).to(torch.bfloat16)
    W_gu = rnd_bf16(g, 2 * d.I_DENSE, d.H, std=0.02)
    W_down = rnd_bf16(g, d.H, d.I_DENSE, std=0.02)
    mid = torch.zeros(2 * d.I_DENSE, dtype=torch.bfloat16, device=DEV)
    act = torch.zeros(d.I_DENSE, dtype=torch.bfloat16, device=DEV)
    h = torch.zeros(d.H, dtype=torch.bfloat16, device=DEV)
    x_res = x.clone()
    ops = [B.gateup_layer(mk, None, x_res, W_gu, act, inter=d.I_DENSE, groups=1, expert=False, norm=True,
                          w_norm=w_norm, mid=mid, h_out=h),
           B.linear_gemv_layer(mk, None, input=act, weight=W_down, output=x_res, residual=x_res, residual_add=True)]
    run_ops(mk, ops)
    hh = R.rmsnorm(np32(x), np32(w_norm))
    mid_w, act_w, out_w = R.dense_mlp(hh, OracleModel.gate_up(np32(W_gu)), np32(W_down), np32(x), d.I_DENSE)
    assert_bits_equal(h, hh, "h")
    assert_bits_equal(mid, mid_w, "mid")
    assert_bits_equal(act, act_w, "act")
    assert_bits_equal(x_res, out_w, "x_res")


def test_wait_timeout_reports_and_recovers(mk, B):
    """Failure detection without a GPU fault: an operator whose wait never succeeds runs into the
    bounded spin, the status word says wait_timeout, and the same handle runs again after reset."""
    g = gen(61)
    W = rnd_bf16(g, 256, 512, std=0.02)
    x = rnd_bf16(g, 512)
    out1 = torch.zeros(256, dtype=torch.bfloat16, device=DEV)
    out2 = torch.zeros(512, dtype=torch.bfloat16, device=DEV)
    W2 = rnd_bf16(g, 512, 256, std=0.02)
    k = mk.MegaKernel(0, wait_timeout_s=0.2)
    k.add(B.linear_gemv_layer(mk, None, input=x, weight=W, output=out1))
    k.add(B.linear_gemv_layer(mk, None, input=out1, weight=W2, output=out2))
    k.finalize()
    k.block_op(1)
    k.launch(1, 0)
    st = k.status(raise_on_error=False)
    assert st["error"] == 1 and st["err_op"] == 1, st          # MK_DERR_WAIT_TIMEOUT at operator 1
    k.reset()
    k.launch(1, 0)
    assert k.status()["error"] == 0
    want1 = R.linear(np32(x), np32(W))
    assert_bits_equal(out1, want1, "out1")
    assert_bits_equal(out2, R.linear(want1, np32(W2)), "out2")


def test_rejects_bad_plans(mk, B):
    k = mk.MegaKernel(0)
    bad = mk.make_op(mk.OP_GEMV, 0, {}, {0: 16, 1: 20})      # K not a multiple of 8, null pointers
    with pytest.raises(mk.MkError):
        k.add(bad)
    with pytest.raises(mk.MkError):
        k.launch(1, 0)                                      # not finalized
