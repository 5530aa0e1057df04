"""Operator-by-operator parity of the decode graph (the reference's --stop-after protocol with its
boundary keys, harness/run_fleet.py:69-147): the plan is truncated after each operator of the first
iteration, and the workspace that operator wrote must equal the oracle's value bit for bit."""
import numpy as np
import pytest
import torch

from gpu_helpers import DeviceWeights, assert_bits_equal, np32
from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

SMALL = dict(H=256, NH=4, D_N=32, D_R=16, D_V=32, D_C=64, V=1024, L=3, I_DENSE=384, I_MOE=64, E=8, TOPK=2, N_SHARED=2)


def _setup(dims, split, seed=0, n_past=40):
    from fleet import build_graph as B
    from fleet.capture import make_capture
    from fleet.pack_weights import synthetic_packed
    s_max = n_past + 3
    packed = synthetic_packed(dims, layers=dims.L, head=True, seed=seed, device=DEV, random_norms=True)
    capture = make_capture(dims, dims.L, s_max, n_past, seed=seed + 1, device=DEV)
    prompt = torch.randint(0, dims.V, (n_past + 1,), generator=torch.Generator().manual_seed(seed + 2)).tolist()
    return packed, capture, prompt, s_max, n_past


def _oracle(dims, packed, capture, prompt, n_past, split):
    from fleet.capture import softmax_scale
    dw = DeviceWeights(packed)
    m = OracleModel(dims, dw.get, dw.get_expert, softmax_scale=softmax_scale(dims.D_N, dims.D_R), split=split)
    cache = {k: np32(v) for k, v in capture.items() if k.startswith(("c_kv_", "k_pe_"))}
    _, _, rec = m.step(prompt[n_past], n_past, cache, np32(capture["cos"]), np32(capture["sin"]), record=True)
    return rec


CHECKS = {   # label suffix -> [(workspace, record key, slice)]
    "qkva": [("qkva", "qkva", None), ("h", "norm1", None)],
    "mla_prep": [("ql_nope", "ql_nope", None), ("q_pe", "q_pe", None)],
    "mla_merge_uv": [("attn", "attn", None)],
    "o_proj": [("x_res", "x_res_attn", None)],
    "gate_up": [("act0", "act", None), ("h", "norm2", None)],
    "down": [("x_res", "layer_out", None)],
    "router": [("h", "norm2", None)],
    "w13s": [("act8", None, None)],
    "w13r": [("act8", None, None)],
    "w2_combine": [("x_res", "layer_out", None), ("out8", "out8", None)],
    "experts": [("act8", None, None)],
    "combine": [("x_res", "layer_out", None), ("out8", "out8", None)],
}


@pytest.mark.parametrize("which,split,moe", [("small", 16, "units"), ("small", 64, "units"), ("small", 16, "staged")])
def test_every_boundary(which, split, moe):
    from fleet import build_graph as B
    from fleet.pack_weights import Dims
    from oracle import numpy_ref as R
    dims = Dims(**SMALL)
    packed, capture, prompt, s_max, n_past = _setup(dims, split)
    rec = _oracle(dims, packed, capture, prompt, n_past, split)
    plan = B.G.build_plan(dims, s_max, dims.L, True, split=split, moe=moe)
    labels = [c.label for c in plan.calls]
    failures = []
    for lab in labels:
        cap = {k: v.clone() for k, v in capture.items()}
        meta = B.make_meta(torch, s_max, prompt, n_past + 1, device=DEV)
        mpk, host, plan2 = B.build(packed, cap, meta, dims=dims, s_max=s_max, layers=dims.L, head=True,
                                   stop_after=lab, split=split, moe=moe)
        mpk.compile()
        mpk.step = n_past - 1
        mpk.launch(1)
        assert mpk.status()["error"] == 0
        torch.cuda.synchronize()
        prefix, op = lab.split(".", 1)
        if prefix == "head":
            checks = [("logits", "head.logits"), ("h", "head.norm")]
        elif prefix == "prologue":
            checks = [("x_res", "embed")]
        else:
            checks = [(ws, f"{prefix}.{key}") for ws, key, _ in CHECKS.get(op, []) if key]
            if op == "mla_prep":
                l = int(prefix[1:])
                got = np32(host[f"c_kv_{l}"][n_past])
                if not np.array_equal(got, rec[f"{prefix}.c_kv"]):
                    failures.append(f"{lab}: c_kv row")
            if op == "mla_attend":
                d_c = dims.D_C
                want = rec[f"{prefix}.partials"]
                got = host["partials"].cpu().numpy()[:, :, :d_c + 1]
                live = -(-(n_past + 1) // split)
                if not np.array_equal(got[:live].view(np.uint32), want[:live].view(np.uint32)):
                    bad = np.nonzero(got[:live] != want[:live])
                    failures.append(f"{lab}: partials differ at {len(bad[0])} places, first {tuple(b[0] for b in bad)}")
            if op in ("w13s", "w13r", "experts"):   # shared slots TOPK.. / routed slots ..TOPK / all of act8
                mask = rec[f"{prefix}.mask"]
                act = np.stack([R.swiglu_act(m, dims.I_MOE) for m in rec[f"{prefix}.mid"][:int(mask[-1])]])
                rows = {"w13s": slice(dims.TOPK, dims.TOPK + dims.N_SHARED), "w13r": slice(0, dims.TOPK),
                        "experts": slice(0, dims.TOPK + dims.N_SHARED)}[op]
                if not np.array_equal(np32(host["act8"])[rows], act[rows]):
                    failures.append(f"{lab}: act8")
                checks = []
        for ws, key in checks:
            got = np32(host[ws]).reshape(-1)
            want = np.asarray(rec[key], np.float32).reshape(-1)[:got.size] if key in rec else None
            if want is None:
                continue
            if got.size != want.size:
                got = got[:want.size]
            if not np.array_equal(got, want):
                bad = np.nonzero(got != want)[0]
                failures.append(f"{lab}: {ws} differs at {bad.size} of {got.size} (first {bad[:4]}: "
                                f"{got[bad[:4]]} vs {want[bad[:4]]})")
        mpk.kernel.close()
    assert not failures, "\n".join(failures)
