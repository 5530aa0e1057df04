"""CPU restatement of the decode step's per-operator math (the reference's NumPy specification,
harness/numpy_ref.py:36-321, plus the stock tasks it composes with: embedding, dense SwiGLU,
combine, argmax).

TEST INFRASTRUCTURE. This module is the checker the CUDA path is compared with; it is never the
thing measured or shipped. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import it.

Rounding points are the reference's (BF16 wherever the reference stores BF16 or feeds a BF16
matrix operand); the two freedoms the reference leaves open are closed as ``oracle.detmath``
explains: every FP32 sum runs in the kernels' specified order, and exp/log are deterministic
routines. So the CUDA kernels must agree bit for bit, and the reference's own functions agree
within their own tolerances (tests/test_oracle_pins.py checks both).

Array conventions: BF16 tensors are float32 arrays holding BF16 values (as numpy_ref does); weights
may also be uint16 arrays of BF16 bit patterns (device tensors copied as 16-bit words), which the
row dots read directly.
"""
import numpy as np

from oracle.detmath import (F32, F64, _od, bf16, block_sum, butterfly, det_exp, det_log, dot_rows, lane_sum,
                            seq_sum, silu, vals)

__all__ = ["bf16", "rmsnorm", "rope", "mla_prep", "mla_attend", "merge_partials", "mla_merge_uv",
           "attention_decompressed",
           "moe_router", "moe_router_norm", "moe_w13", "moe_w2", "silu", "linear", "linear_norm",
           "linear_residual", "moe_combine", "dense_mlp", "embed", "lm_head_argmax",
           "partials_row", "softmax_det", "e4m3", "f16", "linear_fp8", "moe_experts_fp8"]


def partials_row(d_c):
    """Innermost width of the split-KV partials: d_c values of o, the lse at column d_c, padded
    to a multiple of 4 floats (16-byte rows). The reference's layout: fleet/graph_plan.py:214-218."""
    return ((d_c + 1 + 3) // 4) * 4


# ---------------------------------------------------------------------------------------------
# norms and rotary embedding


def rmsnorm(x, w, eps=1e-6):
    """DeepseekV2RMSNorm on BF16 inputs (numpy_ref.py:54-60; modeling_deepseek.py:94-108).
    FP32 sum of squares in the 256-thread block order (detmath.block_sum), divided by n; then
    FP32 1/sqrt(var + eps), the normalised value rounded to BF16, times the BF16 weight, rounded."""
    x = vals(x)
    n = x.shape[-1]
    var = (block_sum((x * x).astype(F32)) / F32(n)).astype(F32)[..., None]
    r = (F32(1.0) / np.sqrt((var + F32(eps)).astype(F32))).astype(F32)
    xn = bf16((x * r).astype(F32))
    return bf16((vals(w) * xn).astype(F32))


def rope(x, cos_row, sin_row):
    """apply_rotary_pos_emb on the last dim (numpy_ref.py:63-71; modeling_deepseek.py:339-372):
    de-interleave (even, odd) pairs into two halves, then bf16(bf16(x cos) + bf16(rot sin)).
    Each rounding follows one FP32 operation on BF16 values, so this is exact on any machine."""
    x = np.asarray(x, F32)
    d = x.shape[-1]
    x = x.reshape(*x.shape[:-1], d // 2, 2).swapaxes(-1, -2).reshape(*x.shape[:-1], d)
    h = d // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return bf16(bf16((x * vals(cos_row)).astype(F32))
                + bf16((rot * vals(sin_row)).astype(F32)))


# ---------------------------------------------------------------------------------------------
# linears (the batch-1 GEMVs)


def linear(x, W):
    """bf16(W x): FP32 accumulation in the kernels' order, one rounding (numpy_ref.py:304-307)."""
    return bf16(dot_rows(W, x))


def linear_residual(x, W, res):
    """bf16(W x + res), the residual added in FP32 before the one rounding (numpy_ref.py:310-313)."""
    return bf16((dot_rows(W, x) + np.asarray(res, F32)).astype(F32))


def linear_norm(x, w_norm, W, eps=1e-6):
    """rmsnorm prologue then the linear (numpy_ref.py:295-301). Returns (h, out)."""
    h = rmsnorm(x, w_norm, eps)
    return h, linear(h, W)


# ---------------------------------------------------------------------------------------------
# MLA


def mla_prep(qkva, w_kv_norm, W_uk, cos_row, sin_row, *, nh=16, d_n=128, d_r=64, d_c=512,
             eps=1e-6):
    """One decode token (numpy_ref.py:85-103; mla_prep_mi300.cuh:34-139).
    qkva [nh*(d_n+d_r) + d_c + d_r]; W_uk [nh, d_n, d_c]. Returns c_row [d_c], k_pe_row [d_r],
    ql_nope [nh, d_c] = bf16(q_nope[h] @ W_uk[h]), q_pe [nh, d_r]."""
    q_out = nh * (d_n + d_r)
    qkva = np.asarray(qkva, F32)
    q = qkva[:q_out].reshape(nh, d_n + d_r)
    c_raw = qkva[q_out:q_out + d_c]
    k_pe_raw = qkva[q_out + d_c:q_out + d_c + d_r]
    c_row = rmsnorm(c_raw, w_kv_norm, eps)
    k_pe_row = rope(k_pe_raw, cos_row, sin_row)
    q_nope, q_pe = q[:, :d_n], q[:, d_n:]
    q_pe = rope(q_pe, cos_row, sin_row)
    W_uk = np.asarray(W_uk)
    ql = np.stack([dot_rows(W_uk[h].T, q_nope[h]) for h in range(nh)])
    return c_row, k_pe_row, bf16(ql), q_pe


def score_lanes(d):
    """Columns per lane of a d-wide score operand: d / 32 contiguous columns when d >= 32 (lane l
    takes [l*n, l*n + n)), else one column for lanes l < d."""
    return max(1, d // 32)


def _scores(ql_nope_h, q_pe_h, c_rows, k_rows):
    """One head's FP32 scores against cache rows, in the kernels' order: lane l adds the products
    of its contiguous latent columns [l*LC, l*LC + LC) in order, then of its contiguous rope
    columns [l*RP, l*RP + RP), into one accumulator; then the butterfly. Products of BF16 values
    are exact. (d_c is a multiple of 32; d_r is a multiple of 32 or below it.)"""
    rows = c_rows.shape[0]
    acc = np.zeros((rows, 32), F32)
    lanes = np.arange(32)
    for cols, q in ((c_rows, ql_nope_h), (k_rows, q_pe_h)):
        d = cols.shape[1]
        n = score_lanes(d)
        for m in range(n):
            col = lanes * n + m
            ok = col < d
            cc = np.minimum(col, d - 1)
            prod = (cols[:, cc] * q[cc]).astype(F32)
            acc = np.where(ok, (acc + prod).astype(F32), acc)
    return butterfly(acc)


def mla_attend(ql_nope, q_pe, c_kv, k_pe, step, softmax_scale, *, split=32, n_splits=None,
               debug_scores=False):
    """Split-KV attention over cache rows [0, step] (numpy_ref.py:110-149).

    Per split j (rows [j*split, min(j*split+split, step+1))) and head h:
      s = (FP32 q.k in the kernels' order) * f32(scale)
      m = max s;  p = det_exp(s - m);  l = FP32 sum of p (one warp: lanes then butterfly)
      o = (FP32 sum over rows, in row order, of bf16(p) c_kv) / l;  lse = m + det_log(l)
    An empty split stores o = 0 and lse = -inf. Returns partials [n_splits, nh, d_c + 1] FP32
    (and the scaled scores [nh, step + 1] with debug_scores)."""
    ql_nope = np.ascontiguousarray(vals(ql_nope))
    q_pe = np.ascontiguousarray(vals(q_pe))
    c_kv = np.ascontiguousarray(vals(c_kv))
    k_pe = np.ascontiguousarray(vals(k_pe))
    nh, d_c = ql_nope.shape
    s_max = c_kv.shape[0]
    n_splits = n_splits or -(-s_max // split)
    partials = np.zeros((n_splits, nh, d_c + 1), F32)
    L = _od()
    if L is not None and not debug_scores and split <= 4096:      # detdot.c: the same operations
        L.od_mla_attend(ql_nope.ctypes.data, q_pe.ctypes.data, c_kv.ctypes.data, k_pe.ctypes.data, nh, d_c,
                        q_pe.shape[1], int(step), F32(softmax_scale), int(split), int(n_splits),
                        partials.ctypes.data)
        return partials
    scores_all = np.zeros((nh, step + 1), F32) if debug_scores else None
    scale = F32(softmax_scale)
    for j in range(n_splits):
        lo, hi = j * split, min(j * split + split, step + 1)
        if lo > step:
            partials[j, :, d_c] = -np.inf
            continue
        for h in range(nh):
            s = (_scores(ql_nope[h], q_pe[h], c_kv[lo:hi], k_pe[lo:hi]) * scale).astype(F32)
            if debug_scores:
                scores_all[h, lo:hi] = s
            m = s.max()
            p = det_exp((s - m).astype(F32))
            l = lane_sum(p)
            acc = seq_sum((bf16(p)[:, None] * c_kv[lo:hi]).astype(F32), axis=0)
            partials[j, h, :d_c] = (acc / l).astype(F32)
            partials[j, h, d_c] = (m + det_log(l)).astype(F32)
    return (partials, scores_all) if debug_scores else partials


def merge_partials(partials, step, *, split=32, d_c=None):
    """Merge of the live splits (numpy_ref.py:152-165): M = max lse, w_j = det_exp(lse_j - M),
    o = (sum_j f32(w_j o_j)) / (sum_j w_j), both sums sequential over j in FP32.
    d_c: the logical width when rows are padded."""
    if d_c is None:
        d_c = partials.shape[2] - 1
    live = -(-(step + 1) // split)
    lse = np.asarray(partials[:live, :, d_c], F32)
    M = lse.max(axis=0)
    with np.errstate(invalid="ignore"):
        w = det_exp((lse - M[None, :]).astype(F32))                    # [live, nh]
    o = np.asarray(partials[:live, :, :d_c], F32)
    num = seq_sum((w[:, :, None] * o).astype(F32), axis=0)
    den = seq_sum(w, axis=0)
    return (num / den[:, None]).astype(F32)


def mla_merge_uv(partials, W_uv, step, *, split=32, d_c=None):
    """attn [nh * d_v]: per head the merge, o rounded to BF16, then bf16(W_uv[h] o[h])
    (numpy_ref.py:168-174)."""
    o = bf16(merge_partials(partials, step, split=split, d_c=d_c))
    W_uv = np.asarray(W_uv)
    attn = np.stack([dot_rows(W_uv[h], o[h]) for h in range(W_uv.shape[0])])
    return bf16(attn.reshape(-1))


def attention_decompressed(q_nope, q_pe, c_kv, k_pe, W_uk, W_uv, step, softmax_scale):
    """The model's own attention order for the same token, with the keys and values decompressed
    (harness/numpy_ref.py:187-198, restated): k_nope = bf16(W_uk c) and v = bf16(W_uv c) per
    position (BF16 like the model's kv_b_proj output), scores q_nope . k_nope + q_pe . k_pe in FP32,
    scaled and rounded to BF16 (the model's attn_weights), an FP32 softmax rounded to BF16, then
    bf16(P v). It bounds the error of the absorbed form (scores against the latent, W_uv after the
    merge), which reassociates these products. Returns (attn [nh * d_v], scores [nh, step + 1])."""
    c = vals(c_kv)[:step + 1].astype(F32)
    W_uk, W_uv = vals(W_uk), vals(W_uv)
    k_nope = bf16(np.einsum("hnc,sc->hsn", W_uk, c, dtype=F32, optimize=True))
    v = bf16(np.einsum("hvc,sc->hsv", W_uv, c, dtype=F32, optimize=True))
    s = np.einsum("hn,hsn->hs", vals(q_nope), k_nope, dtype=F32, optimize=True)
    s = (s + vals(q_pe) @ vals(k_pe)[:step + 1].T).astype(F32)
    s = bf16((s * F32(softmax_scale)).astype(F32))
    e = np.exp((s - s.max(axis=-1, keepdims=True)).astype(F32)).astype(F32)
    p = bf16((e / e.sum(axis=-1, keepdims=True)).astype(F32))
    out = np.einsum("hs,hsv->hv", p, v, dtype=F32, optimize=True)
    return bf16(out.reshape(-1)), s


# ---------------------------------------------------------------------------------------------
# MoE


def softmax_det(logits):
    """FP32 softmax with the deterministic exp: e = det_exp(l - max l), p = e / (one warp's FP32
    sum of e: lane l adds experts l, l + 32, ..., then the butterfly)."""
    logits = np.asarray(logits, F32)
    m = logits.max(axis=-1, keepdims=True)
    e = det_exp((logits - m).astype(F32))
    s = lane_sum(e)[..., None]
    return (e / s).astype(F32)


def moe_router(h, W_gate, *, topk=6, n_experts=64, forced=(64, 65), scaling=1.0, logit_bias=None):
    """FP32 router with the shared experts forced in (numpy_ref.py:205-234;
    moe_router_mi300.cuh:115-354; HF MoEGate modeling_deepseek.py:393-470).

    logits = f32(exact W_gate h) (+ logit_bias, FP32, when given: the injected-routing case);
    p = softmax; top-k by repeated argmax, ties to the lower index; topk_w = p * scaling, then
    1.0 per forced expert; routing [E + n_forced] (slot + 1, else 0); mask [E + n_forced + 1]
    (ids in slot order, -1 in unused entries, the count last)."""
    logits = dot_rows(W_gate, h)
    if logit_bias is not None:
        logits = (logits + np.asarray(logit_bias, F32)).astype(F32)
    p = softmax_det(logits)
    idx = []
    remaining = p.copy()
    for _ in range(topk):
        e = int(np.argmax(remaining))
        idx.append(e)
        remaining[e] = -np.inf
    ids = idx + list(forced)
    n_slots = topk + len(forced)
    n_total = n_experts + len(forced)
    topk_w = np.array([p[e] * F32(scaling) for e in idx] + [1.0] * len(forced), F32)
    routing = np.zeros(n_total, np.int32)
    for k, e in enumerate(ids):
        routing[e] = k + 1
    mask = np.full(n_total + 1, -1, np.int32)
    mask[:n_slots] = ids
    mask[n_total] = n_slots
    return logits, topk_w, routing, mask


def moe_router_norm(x_res, w_norm, W_gate, *, eps=1e-6, topk=6, n_experts=64, forced=(64, 65),
                    scaling=1.0, logit_bias=None):
    """The router with the post-attention norm folded in (numpy_ref.py:237-245).
    Returns (h, logits, topk_w, routing, mask)."""
    h = rmsnorm(x_res, w_norm, eps)
    return (h,) + moe_router(h, W_gate, topk=topk, n_experts=n_experts, forced=forced,
                             scaling=scaling, logit_bias=logit_bias)


def moe_w13(h, W13, mask, n_slots=8):
    """mid[s] = bf16(W13[mask[s]] h) for the active slots, NaN rows past the count
    (numpy_ref.py:256-272). W13 [E, 2I, H] (gate rows then up rows)."""
    n_active = int(mask[-1])
    mid = np.full((n_slots, np.shape(W13)[1]), np.nan, F32)
    for s in range(n_active):
        mid[s] = linear(h, W13[int(mask[s])])
    return mid


def swiglu_act(mid_row, i):
    """act = bf16(silu(gate) * up) element by element (numpy_ref.py:288-290)."""
    mid_row = np.asarray(mid_row, F32)
    return bf16((silu(mid_row[:i]) * mid_row[i:2 * i]).astype(F32))


def moe_w2(mid, W2, mask, n_slots=8):
    """out8[s] = bf16(W2[e] act_s), act_s = bf16(silu(gate) * up) (numpy_ref.py:275-292)."""
    k = np.shape(W2)[2]
    n_active = int(mask[-1])
    out = np.full((n_slots, np.shape(W2)[1]), np.nan, F32)
    for s in range(n_active):
        out[s] = linear(swiglu_act(mid[s], k), W2[int(mask[s])])
    return out


def moe_combine(out8, topk_w, x_res):
    """x + sum_k w_k out_k in slot order, FP32 products and sums each rounded, then BF16: the
    exact operation sequence of numpy_ref.py:316-321 (the stock moe_mul_sum_add)."""
    acc = np.asarray(x_res, F32).copy()
    for k in range(len(topk_w)):
        acc = (acc + (np.asarray(out8[k], F32) * F32(topk_w[k])).astype(F32)).astype(F32)
    return bf16(acc)


def dense_mlp(h, W_gu, W_down, x_res, i_dense):
    """Layer 0's SwiGLU MLP (stock gang_linear_silu + linear_with_residual, plan
    fleet/graph_plan.py:507-526), with the expert arithmetic: mid = bf16(W_gu h) [gate; up],
    act = bf16(silu(gate) * up), x_res = bf16(W_down act + x_res). Returns (mid, act, x_res)."""
    mid = linear(h, W_gu)
    act = swiglu_act(mid, i_dense)
    return mid, act, linear_residual(act, W_down, x_res)


# ---------------------------------------------------------------------------------------------
# prologue and head


def embed(W_embed, token):
    """x_res = W_embed[token] (the stock embedding task, fleet/graph_plan.py:416-418)."""
    return vals(W_embed[int(token)]).copy()


def lm_head_argmax(x_res, w_final_norm, W_lm, eps=1e-6):
    """h = rmsnorm(x_res); logits = bf16(W_lm h); token = argmax, lowest index on ties
    (fleet/graph_plan.py:570-602; torch.argmax as harness/run_reference.py:395 uses it).
    Returns (h, logits, token)."""
    h = rmsnorm(x_res, w_final_norm, eps)
    logits = linear(h, W_lm)
    return h, logits, int(np.argmax(logits))


# ---------------------------------------------------------------------------------------------
# FP8 weight-only experts (the reference's D26 plan, docs/acceleration/01-precision.md:125-165:
# E4M3 weights with a per-tensor scale, BF16 activations, FP32 accumulation; no FP8 kernel of the
# reference exists, so the arithmetic below is this build's specified form)


def e4m3_table():
    """float32 value of every E4M3 byte (OCP FP8 E4M3FN: bias 7, subnormals m * 2^-9, 0x7F / 0xFF
    NaN, no infinity), from the format's definition."""
    t = np.empty(256, F32)
    for b in range(256):
        s, e, m = b >> 7, (b >> 3) & 15, b & 7
        if e == 15 and m == 7:
            v = np.nan
        elif e == 0:
            v = m * 2.0 ** -9
        else:
            v = (1.0 + m / 8.0) * 2.0 ** (e - 7)
        t[b] = -v if s else v
    return t


_E4M3 = None


def e4m3(q):
    """uint8 E4M3 codes -> float32 values (exact)."""
    global _E4M3
    if _E4M3 is None:
        _E4M3 = e4m3_table()
    return _E4M3[np.asarray(q, np.uint8)]


def f16(x):
    """float32 values rounded to FP16 (nearest even) and back, finite values beyond the FP16 range
    saturated at +-65504: the FP8 path's activation operand."""
    x = np.asarray(x, F32)
    with np.errstate(over="ignore"):
        y = x.astype(np.float16).astype(F32)
    return np.where(np.isinf(y) & np.isfinite(x), np.copysign(F32(65504.0), x), y).astype(F32)


def linear_fp8(x, Wq, scale):
    """bf16(scale * (E4M3 rows . fp16(x))): each product of an E4M3 value (4 significant bits) and an
    FP16 value (11) is exact in FP32, the sum runs in the row-dot order, one FP32 multiply by the
    tensor's scale, one BF16 rounding."""
    return bf16((F32(scale) * dot_rows(e4m3(Wq), f16(x))).astype(F32))


def moe_experts_fp8(h, W13q, s13, W2q, s2, mask, n_slots=8):
    """The experts with E4M3 weights: per slot s (expert e = mask[s]) gate = linear_fp8(h, rows 2i of
    W13q[e], s13[e, 0]), up likewise with rows 2i + 1 and s13[e, 1], act = bf16(silu(gate) up),
    out8[s] = linear_fp8(act, W2q[e], s2[e]). W13q [E, 2I, H] (gate and up interleaved), W2q
    [E, H, I], uint8. Returns (act [n_slots, I], out8 [n_slots, H])."""
    W13q = np.asarray(W13q)
    I = W13q.shape[1] // 2
    act = np.full((n_slots, I), np.nan, F32)
    out8 = np.full((n_slots, np.shape(W2q)[1]), np.nan, F32)
    for s in range(int(mask[-1])):
        e = int(mask[s])
        g = linear_fp8(h, W13q[e][0::2], s13[e][0])
        u = linear_fp8(h, W13q[e][1::2], s13[e][1])
        act[s] = swiglu_act(np.concatenate([g, u]), I)
        out8[s] = linear_fp8(act[s], W2q[e], s2[e])
    return act, out8
