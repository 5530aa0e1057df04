"""End-to-end parity of the persistent decode graph with the CPU oracle (oracle/model.py).

The graph is built through the reference-shaped surface (fleet/build_graph.build with the packed
weights, the capture and the meta tensors), runs greedy iterations in one launch, and must give
the oracle's token ids, route log, cache rows and final residual bit for bit. DeepSeek-V2-Lite
shapes with a reduced layer count (layer 0 dense + MoE layers + the head) so the oracle finishes
in seconds; the full 27-layer graph is the bench's workload.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import DeviceFP8, DeviceWeights, assert_bits_equal, np32
from oracle.detmath import from_bf16_bits
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def build_model(layers, iters, n_past=1023, seed=0, random_norms=True, dims=None, split=None, moe=None):
    from fleet import build_graph as B
    from fleet import graph_plan as G
    from fleet.capture import make_capture
    from fleet.pack_weights import REAL_DIMS, synthetic_packed
    d = dims or REAL_DIMS
    s_max = n_past + 1 + iters          # tokens[n_past + 1 .. n_past + iters] are generated
    packed = synthetic_packed(d, layers=layers, head=True, seed=seed, device=DEV, random_norms=random_norms)
    capture = make_capture(d, layers, s_max, n_past, seed=seed + 1, device=DEV)
    prompt = torch.randint(0, d.V, (n_past + 1,), generator=torch.Generator().manual_seed(seed + 2))
    meta = B.make_meta(torch, s_max, prompt.tolist(), n_past + 1, device=DEV)
    cache0 = {k: np32(v) for k, v in capture.items() if k.startswith(("c_kv_", "k_pe_"))}
    kw = {} if split is None else dict(split=split)
    if moe is not None:
        kw["moe"] = moe
    mpk, host, plan = B.build(packed, capture, meta, dims=d, s_max=s_max, layers=layers, head=True, **kw)
    return d, packed, capture, meta, cache0, mpk, host, plan, n_past


def oracle_run(d, packed, capture, meta, cache0, plan, layers, iters, pos0):
    from fleet.capture import softmax_scale
    dw = DeviceWeights(packed)
    m = OracleModel(d, dw.get, dw.get_expert, softmax_scale=softmax_scale(d.D_N, d.D_R), split=plan.split,
                    layers=layers, fp8=DeviceFP8(packed) if plan.moe == "units_fp8" else None)
    tokens = meta["tokens"][0].cpu().numpy().copy()
    cache = {k: v.copy() for k, v in cache0.items()}
    cos, sin = np32(capture["cos"]), np32(capture["sin"])
    ids, routes, rec = m.generate(tokens, pos0, iters, cache, cos, sin, record_last=True)
    return ids, routes, rec, cache


@pytest.mark.parametrize("layers,iters", [(3, 4)])
def test_decode_one_launch_matches_oracle(layers, iters):
    d, packed, capture, meta, cache0, mpk, host, plan, pos0 = build_model(layers, iters)
    mpk.compile()
    meta["step"].fill_(pos0 - 1)
    mpk()                                                    # every remaining iteration, one launch
    st = mpk.status()
    assert st["error"] == 0, st
    assert int(meta["step"].item()) == pos0 - 1 + (plan.s_max - 2 - (pos0 - 1))
    n_run = plan.s_max - 2 - (pos0 - 1)
    ids = meta["tokens"][0, pos0 + 1: pos0 + 1 + n_run].tolist()
    want_ids, routes, rec, cache = oracle_run(d, packed, capture, meta, cache0, plan, layers, n_run, pos0)
    assert ids == want_ids
    rl = host["route_log"].cpu().numpy()
    for i in range(n_run):
        for l in range(1, layers):
            assert rl[i, l - 1, :d.TOPK].tolist() == routes[i][l - 1], (i, l)
    for l in range(layers):
        got = host[f"c_kv_{l}"][pos0:pos0 + n_run].float().cpu().numpy()
        assert np.array_equal(got, cache[f"c_kv_{l}"][pos0:pos0 + n_run]), l
        got = host[f"k_pe_{l}"][pos0:pos0 + n_run].float().cpu().numpy()
        assert np.array_equal(got, cache[f"k_pe_{l}"][pos0:pos0 + n_run]), l
    # the last iteration's workspaces: the final residual, the logits and the last layer's router
    assert_bits_equal(host["logits"][0], rec["head.logits"], "logits")
    assert_bits_equal(host["h"][0], rec["head.norm"], "final norm")
    L = layers - 1
    assert np.array_equal(host["mask"].cpu().numpy(), rec[f"L{L}.mask"])
    assert_bits_equal(host["out8"], rec[f"L{L}.out8"], "out8")


def test_decode_fp8_experts_matches_oracle():
    """The FP8-expert graph (moe="units_fp8": E4M3 expert weights quantised per tensor from the
    BF16 checkpoint, fleet_mk.h MK_F_FP8): a dense layer, two MoE layers and the head, three greedy
    iterations in one launch; ids, route log, cache rows, logits and out8 equal the oracle running
    the same FP8 experts bit for bit."""
    layers = 3
    d, packed, capture, meta, cache0, mpk, host, plan, pos0 = build_model(layers, 3, seed=3, moe="units_fp8")
    assert plan.moe == "units_fp8" and "W13_1" not in host and host["W13Q_1"].dtype == torch.uint8
    mpk.compile()
    meta["step"].fill_(pos0 - 1)
    mpk()
    assert mpk.status()["error"] == 0
    n_run = plan.s_max - 2 - (pos0 - 1)
    ids = meta["tokens"][0, pos0 + 1: pos0 + 1 + n_run].tolist()
    want_ids, routes, rec, cache = oracle_run(d, packed, capture, meta, cache0, plan, layers, n_run, pos0)
    assert ids == want_ids
    rl = host["route_log"].cpu().numpy()
    for i in range(n_run):
        for l in range(1, layers):
            assert rl[i, l - 1, :d.TOPK].tolist() == routes[i][l - 1], (i, l)
    for l in range(layers):
        got = host[f"c_kv_{l}"][pos0:pos0 + n_run].float().cpu().numpy()
        assert np.array_equal(got, cache[f"c_kv_{l}"][pos0:pos0 + n_run]), l
    assert_bits_equal(host["logits"][0], rec["head.logits"], "logits")
    assert_bits_equal(host["out8"], rec[f"L{layers - 1}.out8"], "out8")


def test_decode_launch_per_token_equals_one_launch():
    """Three launches of one iteration give the same ids and state as one launch of three."""
    layers, iters = 2, 3
    d, packed, capture, meta, cache0, mpk, host, plan, pos0 = build_model(layers, iters, seed=5)
    mpk.compile()
    mpk.step = pos0 - 1
    for _ in range(plan.s_max - 2 - (pos0 - 1)):
        mpk.launch(1)
    assert mpk.status()["error"] == 0
    n_run = plan.s_max - 2 - (pos0 - 1)
    ids = meta["tokens"][0, pos0 + 1: pos0 + 1 + n_run].tolist()
    want_ids, _, rec, _ = oracle_run(d, packed, capture, meta, cache0, plan, layers, n_run, pos0)
    assert ids == want_ids
    assert_bits_equal(host["logits"][0], rec["head.logits"], "logits")


def test_launch_rejects_positions_past_the_cache():
    """A launch whose iterations would append cache rows or write tokens at s_max or beyond (or a
    step below -1) is refused before anything runs; the handle still decodes afterwards."""
    from fleet import mk
    layers, iters = 2, 2
    d, packed, capture, meta, cache0, mpk, host, plan, pos0 = build_model(layers, iters, seed=9)
    mpk.compile()
    for step, n in ((plan.s_max - 2, 1), (plan.s_max - 4, 3), (-2, 1)):
        with pytest.raises(mk.MkError, match="s_max|step"):
            mpk.kernel.launch(n, step)
    tok = torch.zeros(1, dtype=torch.int64, pin_memory=True)
    with pytest.raises(mk.MkError, match="s_max"):
        mpk.kernel.decode_token(meta["tokens"][0], plan.s_max - 2, tok, tok)
    mpk.step = pos0 - 1
    mpk.launch(plan.s_max - 2 - (pos0 - 1))             # the last position is s_max - 1: allowed
    assert mpk.status()["error"] == 0


def test_decode_token_host_to_host():
    """mk_decode_token (the end-to-end call): each step copies the host's token in, decodes one
    token and copies it out; the host-fed greedy ids equal the oracle's. The device row holds no
    token the host did not send (the prompt's last token is cleared there first)."""
    layers, iters = 2, 3
    d, packed, capture, meta, cache0, mpk, host, plan, pos0 = build_model(layers, iters, seed=7)
    mpk.compile()
    mpk.step = pos0 - 1
    tok_in = torch.zeros(1, dtype=torch.int64, pin_memory=True)
    tok_out = torch.zeros(1, dtype=torch.int64, pin_memory=True)
    first = int(meta["tokens"][0, pos0].item())
    tok_in.fill_(first)
    meta["tokens"][0, pos0:] = -1
    n_run = plan.s_max - 2 - (pos0 - 1)
    ids = []
    for _ in range(n_run):
        mpk.decode_token(tok_in, tok_out)
        ids.append(int(tok_out.item()))
        tok_in.copy_(tok_out)
    assert mpk.status()["error"] == 0
    meta["tokens"][0, pos0] = first
    want_ids, _, _, _ = oracle_run(d, packed, capture, meta, cache0, plan, layers, n_run, pos0)
    assert ids == want_ids


def test_decode_8k_context_matches_oracle():
    """Config 4's context on one GPU: 8,191 cached rows (seed 5), so every layer's attention runs
    65 splits of 128 rows per head and the merge combines all of them; a dense layer and a MoE
    layer, two greedy iterations in one launch, bit for bit against the oracle."""
    layers, iters = 2, 2
    d, packed, capture, meta, cache0, mpk, host, plan, pos0 = build_model(layers, iters, n_past=8191, seed=4)
    assert plan.n_splits >= 65
    mpk.compile()
    meta["step"].fill_(pos0 - 1)
    mpk()
    st = mpk.status()
    assert st["error"] == 0, st
    ids = meta["tokens"][0, pos0 + 1: pos0 + 1 + iters].tolist()
    want_ids, routes, rec, cache = oracle_run(d, packed, capture, meta, cache0, plan, layers, iters, pos0)
    assert ids == want_ids
    rl = host["route_log"].cpu().numpy()
    for i in range(iters):
        assert rl[i, 0, :d.TOPK].tolist() == routes[i][0], i
    for l in range(layers):
        got = host[f"c_kv_{l}"][pos0:pos0 + iters].float().cpu().numpy()
        assert np.array_equal(got, cache[f"c_kv_{l}"][pos0:pos0 + iters]), l
    assert_bits_equal(host["logits"][0], rec["head.logits"], "logits")
