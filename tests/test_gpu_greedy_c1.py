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
    assert plan.n_ops == 243 and plan.layers == 27
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


def test_c1_tensor_core_attention_within_tolerance(c1):
    """The same decode with the MLA attention on the tensor cores (FP32 accumulation in the tensor
    cores' order, so every attention output differs from the specified-order one in the last bits
    and the differences compound over 27 layers and 32 steps). Step 0 starts from the oracle's
    state, so it is held to the north-star tolerance: every cache row it appends within 2e-2 of
    the oracle's (rel_err, the reference's boundary metric), every routed-expert choice equal or a
    tie by the reference's rule (one expert swapped for one whose oracle probability is within 2e-2
    of the larger, harness/compare.py:181-236), the first token equal. Later steps decode from the
    form's own state: how many ids still match is reported, not required (on this random-weight
    model near-ties make greedy ids fragile under any change of summation order; the exact form,
    the default, matches all 32)."""
    from oracle.detmath import from_bf16_bits
    got = run_c1(c1, attend_tc=True)
    pos0, d = c1["w"].first_pos, c1["w"].dims
    worst = 0.0
    for k, v in got["cache"].items():
        g = from_bf16_bits(v[pos0]).astype(np.float64)
        o = c1["ocache"][k][pos0].astype(np.float64)
        rel = float(np.linalg.norm(g - o) / max(np.linalg.norm(o), 1e-30))
        worst = max(worst, rel)
        assert rel <= 2e-2, f"{k}: the step-0 cache row differs by rel_err {rel:.3g}"
    ties = 0
    for j in range(d.L - 1):
        r, f = sorted(c1["routes"][0][j]), sorted(got["route_log"][0, j, :d.TOPK].tolist())
        if r != f:
            gone, new = sorted(set(r) - set(f)), sorted(set(f) - set(r))
            p = c1["margins"][0]["probs"][j + 1]
            assert len(gone) == 1 and abs(float(p[gone[0]]) - float(p[new[0]])) <= 2e-2 * max(p[gone[0]], p[new[0]]), \
                f"MoE layer {j + 1}: routes {f} vs {r} at step 0 is no tie"
            ties += 1
    assert got["ids"][0] == c1["ids"][0]
    first = next((i for i in range(ITERS) if got["ids"][i] != c1["ids"][i]), ITERS)
    print(f"c1 tensor cores: step 0 within tolerance (worst cache row rel_err {worst:.3g}, {ties} route ties); "
          f"ids equal for {first} of {ITERS} steps"
          + (f" (the oracle's top-2 logit gap at step {first}: {c1['margins'][first]['gap']:.3g} of the largest)"
             if first < ITERS else ""))
