"""The north-star check: the full 27-layer DeepSeek-V2-Lite-shaped model (config 1: seeded
synthetic weights, a 1024-token prompt, a seeded latent cache standing in for the prefill) decodes
32 greedy tokens in ONE launch of the persistent kernel, and every token id, every routed-expert
choice of every MoE layer, every latent-cache row the decode appends (27 layers x 32 positions) and
the last token's logits equal the CPU oracle's own 32-step greedy decode from the same initial
state, bit for bit.

The reference runs this loop in harness/run_reference.py:380-398 (torch.argmax, lowest index on
ties, :395) and judges ids and routes with harness/compare.py:161 (compare_ids) and :181-236
(compare_route_log); here the oracle is the reference's NumPy arithmetic in the kernels' specified
summation orders, so the comparison is exact rather than within tolerance.

The oracle's ids are also compared with the committed list tests/golden/c1_greedy_ids.json, which
tests/golden/make_c1_ids.py wrote from the oracle alone on a B200 box (the weights are drawn by the
CUDA generator), and which bench.py checks its timed tokens against.
"""
import json
import time
from pathlib import Path

import numpy as np
import pytest
import torch

from gpu_helpers import DeviceWeightBits, u16
from oracle import numpy_ref as R
from oracle.detmath import bf16_bits
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ITERS = 32
GOLDEN = Path(__file__).resolve().parent / "golden" / "c1_greedy_ids.json"


def oracle_greedy(w, pos0, iters, cache_bits, cos, sin, tokens, margins=None):
    """The oracle's own greedy decode of `iters` tokens from position pos0 (its own cache).
    margins (a list): per iteration, the logit gap between the best and second token relative to
    the largest |logit|, and per MoE layer the router probabilities (for the tie rule)."""
    from fleet.capture import softmax_scale
    from fleet.graph_plan import SPLIT
    d = w.dims
    dw = DeviceWeightBits(w.packed, keep_experts=range(d.E, d.E_TOTAL))
    m = OracleModel(d, dw.get, dw.get_expert, softmax_scale=softmax_scale(d.D_N, d.D_R), split=SPLIT)
    cache = {k: (v.astype(np.uint32) << 16).view(np.float32) for k, v in cache_bits.items()}
    tokens = tokens.copy()
    def note(i, r):
        if margins is not None:
            lg = r["head.logits"].astype(np.float64)
            top2 = np.sort(lg)[-2:]
            probs = {l: R.softmax_det(r[f"L{l}.router_logits"]) for l in range(1, d.L)}
            margins.append(dict(gap=float((top2[1] - top2[0]) / np.abs(lg).max()), probs=probs))

    ids, routes, rec = m.generate(tokens, pos0, iters, cache, cos, sin, record_last=True, on_step=note)
    return ids, routes, rec, cache


@pytest.fixture(scope="module")
def c1():
    """Config 1's workload on the device and the oracle's own 32-step greedy decode of it."""
    from fleet import build_graph as B
    from fleet.workload import greedy_decode
    w = greedy_decode(DEV, new_tokens=ITERS)
    cache0 = {k: u16(v) for k, v in w.capture.items() if k.startswith(("c_kv_", "k_pe_"))}
    meta = B.make_meta(torch, w.s_max, w.prompt, w.n_prompt, device=DEV)
    t0 = time.time()
    cos, sin = (w.capture[k].float().cpu().numpy() for k in ("cos", "sin"))
    tokens = meta["tokens"][0].cpu().numpy().copy()
    margins = []
    ids, routes, rec, ocache = oracle_greedy(w, w.first_pos, ITERS, cache0, cos, sin, tokens, margins)
    if GOLDEN.exists():
        assert ids == json.loads(GOLDEN.read_text())["ids"], "the oracle's ids moved from the committed list"
    return dict(w=w, cache0=cache0, ids=ids, routes=routes, rec=rec, ocache=ocache, oracle_s=time.time() - t0,
                margins=margins)


def run_c1(c1, **build_kw):
    """One launch of all 32 iterations from the workload's initial state."""
    from fleet import build_graph as B
    w = c1["w"]
    d = w.dims
    for k, v in c1["cache0"].items():            # the initial cache (an earlier run appended rows)
        w.capture[k].view(torch.int16).copy_(torch.from_numpy(v.view(np.int16)))
    meta = B.make_meta(torch, w.s_max, w.prompt, w.n_prompt, device=DEV)
    mpk, host, plan = B.build(w.packed, w.capture, meta, dims=d, s_max=w.s_max, layers=d.L, head=True, **build_kw)
    mpk.compile()
    assert plan.n_ops == (217 if plan.moe == "units" else 243) and plan.layers == 27
    mpk()                                        # all 32 iterations in one launch
    st = mpk.status()
    assert st["error"] == 0 and st["launches"] == 1 and st["generation"] == ITERS, st
    out = dict(ids=meta["tokens"][0, w.n_prompt:w.n_prompt + ITERS].tolist(),
               route_log=host["route_log"].cpu().numpy(),             # [32, L - 1, 8], row = iteration
               cache={k: u16(w.capture[k]) for k in c1["cache0"]}, logits=u16(host["logits"][0]))
    mpk.kernel.close()
    return out


def check_routes(c1, got):
    d = c1["w"].dims
    for i in range(ITERS):
        for j in range(d.L - 1):
            r = got["route_log"][i, j, :d.TOPK].tolist()
            assert r == c1["routes"][i][j], f"iteration {i}, MoE layer {j + 1}: routes {r} != {c1['routes'][i][j]}"
        assert got["route_log"][i, :, d.TOPK:].tolist() == [list(range(d.E, d.E_TOTAL))] * (d.L - 1)


def test_c1_27_layers_32_greedy_tokens_one_launch_match_oracle(c1):
    got = run_c1(c1)
    pos0 = c1["w"].first_pos
    assert got["ids"] == c1["ids"], f"greedy ids differ: got {got['ids']}, oracle {c1['ids']}"
    check_routes(c1, got)
    for k, v in got["cache"].items():
        rows = slice(pos0, pos0 + ITERS)
        bad = np.nonzero(v[rows] != bf16_bits(c1["ocache"][k][rows]))
        assert bad[0].size == 0, f"{k}: {bad[0].size} cache values differ (first rows {bad[0][:4] + pos0})"
    assert np.array_equal(got["logits"], bf16_bits(c1["rec"]["head.logits"])), "last token's logits differ"
    print(f"c1 exact: 32 greedy ids equal the oracle's ({c1['oracle_s']:.0f} s of oracle); ids {got['ids']}")


def max_abs_rel(g, o):
    """max |g - o| / max |o| (the per-layer-output metric the tolerance is stated in)."""
    g, o = np.asarray(g, np.float64), np.asarray(o, np.float64)
    return float(np.abs(g - o).max() / max(np.abs(o).max(), 1e-30))


def test_c1_tensor_core_attention_per_layer_tolerance(c1):
    """The same model with the MLA attention on the tensor cores (FP32 accumulation in the tensor
    cores' order: every attention output differs from the specified-order one in the last bits).
    Each layer is held to the tolerance on the input the kernel gave it: one decode step with the
    per-layer residual snapshots (the reference's debug graph) and, per layer l, the oracle's layer l
    applied to the kernel's layer l - 1 output. Then, per layer:
      * the latent-cache row it appends equals the oracle's bit for bit (norm1, q/kv_a and the prep
        come before the attention);
      * the routed experts equal the oracle's, or differ by one tie under the reference's rule
        (harness/compare.py:181-236: the two probabilities within 2e-2 of the larger);
      * the layer output is within max-abs relative error 2e-2 of the oracle's (where the routes
        are equal);
    and the head's logits and token equal the oracle's on the kernel's last residual.
    A 32-step decode then runs from the form's own state; how many ids stay equal to the exact
    oracle's is printed, not required: on this random-weight model the residual stream amplifies
    any difference layer over layer, and near-ties make later greedy ids fragile under any change
    of summation order (the exact form, the default, matches all 32)."""
    from fleet import build_graph as B
    from fleet.capture import softmax_scale
    from fleet.graph_plan import SPLIT
    from oracle.detmath import from_bf16_bits
    w = c1["w"]
    d = w.dims
    pos = w.first_pos
    for k, v in c1["cache0"].items():
        w.capture[k].view(torch.int16).copy_(torch.from_numpy(v.view(np.int16)))
    meta = B.make_meta(torch, w.s_max, w.prompt, w.n_prompt, device=DEV)
    mpk, host, plan = B.build(w.packed, w.capture, meta, dims=d, s_max=w.s_max, layers=d.L, head=True, debug=True,
                              attend_tc=True)
    mpk.compile()
    mpk.launch(1)
    torch.cuda.synchronize()
    st = mpk.status()
    assert st["error"] == 0 and st["generation"] == 1, st
    xs = [from_bf16_bits(u16(host[f"dbg_x_res_{l}"][0])) for l in range(d.L)]
    rows = {k: u16(w.capture[k])[pos].copy() for k in c1["cache0"]}
    routes = host["route_log"].cpu().numpy()[0]
    logits = u16(host["logits"][0])
    token = int(meta["tokens"][0, pos + 1])
    mpk.kernel.close()

    dw = DeviceWeightBits(w.packed, keep_experts=range(d.E, d.E_TOTAL))
    m = OracleModel(d, dw.get, dw.get_expert, softmax_scale=softmax_scale(d.D_N, d.D_R), split=SPLIT)
    cache = {k: from_bf16_bits(v).copy() for k, v in c1["cache0"].items()}
    cos, sin = (w.capture[k].float().cpu().numpy() for k in ("cos", "sin"))
    x_in = R.embed(dw.get("W_embed"), int(meta["tokens"][0, pos]))
    worst, ties = (0.0, -1), 0
    for l in range(d.L):
        rec = {}
        xa = m.attention(l, x_in, cache, cos, sin, pos, rec)
        out = m.dense_mlp(xa, rec) if l == 0 else m.moe(l, xa, rec)
        for k in (f"c_kv_{l}", f"k_pe_{l}"):
            assert np.array_equal(rows[k], bf16_bits(cache[k][pos])), f"{k}: the appended row differs"
        same_route = True
        if l >= 1:
            r, f = sorted(rec[f"L{l}.mask"][:d.TOPK].tolist()), sorted(routes[l - 1, :d.TOPK].tolist())
            if r != f:
                gone, new = sorted(set(r) - set(f)), sorted(set(f) - set(r))
                p = R.softmax_det(rec[f"L{l}.router_logits"])
                assert len(gone) == 1 and abs(float(p[gone[0]]) - float(p[new[0]])) <= \
                    2e-2 * max(p[gone[0]], p[new[0]]), f"layer {l}: routes {f} vs {r} is no tie"
                ties += 1
                same_route = False
        if same_route:
            e = max_abs_rel(xs[l], out)
            assert e <= 2e-2, f"layer {l}: output max-abs relative error {e:.3g}"
            worst = max(worst, (e, l))
        x_in = xs[l]                 # the next layer starts from the kernel's output
    h, ologits, otok = R.lm_head_argmax(xs[-1], dw.get("w_final_norm"), dw.get("W_lm"))
    assert np.array_equal(logits, bf16_bits(ologits)) and token == otok

    got = run_c1(c1, attend_tc=True)
    first = next((i for i in range(ITERS) if got["ids"][i] != c1["ids"][i]), ITERS)
    print(f"c1 tensor cores: per-layer max-abs relative error at most {worst[0]:.3g} (layer {worst[1]}), "
          f"{ties} route ties, cache rows and head exact on the kernel's inputs; a 32-step decode from "
          f"its own state keeps the oracle's ids for {first} of {ITERS} steps"
          + (f" (the oracle's top-2 logit gap at step {first}: {c1['margins'][first]['gap']:.3g} of the largest)"
             if first < ITERS else ""))
