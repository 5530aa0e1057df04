"""Names and numbers shared by the run driver (run_fleet.py), the comparison (compare.py) and the
reference side that writes the files they read.

The boundary keys are the join between a reference run and a run of this package: the same keys,
boundary ids and classes as the reference's harness/common.py:9-106, so a dump of either side can
be compared with the other's. The class thresholds are the reference's starting values on
rel_err (its docs/design-doc/07-correctness.md), replaced by THRESHOLD_MULTIPLIER x the calibrated
floor when a calibration.json is present.
"""
from pathlib import Path

HARNESS = Path(__file__).resolve().parent
PACKAGE = HARNESS.parent

N_PROMPT = 1024
N_STEPS = 32
S_MAX = N_PROMPT + N_STEPS
HANDOVER = N_PROMPT - 1            # the first decode iteration runs at this position
SOFTMAX_SCALE = 0.1147213867929261
BOUNDARY_LAYERS = (0, 1)           # the layers a reference run captures at decode step 0
THRESHOLD_MULTIPLIER = 4.0

CLASS_THRESHOLD = dict(norm=1e-2, rope=1e-2, gemv=2e-2, scores=3e-2, attention=3e-2, router=2e-2,
                       expert=3e-2, layer=5e-2, logits=5e-2, exact=0.0)

# per-layer keys are "L{l}.<suffix>" (an expert key carries its expert id: "L{l}.B11.expert_{e}")
_LAYER = {"B1.norm1": "norm", "B2.q": "gemv", "B3.c_kv": "norm", "B3.k_pe": "rope", "B4.q_pe": "rope",
          "B5.scores": "scores", "B6.attn": "attention", "B7.x_res_attn": "gemv", "B8.router_logits": "router",
          "B9.topk_idx": "exact", "B10.topk_w": "router", "B11.expert_*": "expert", "B12.shared": "expert",
          "B13.layer_out": "layer"}
_HEAD = {"head.B14.norm": "norm", "head.B15.logits": "logits", "head.B16.token": "exact"}
LAYER_BOUNDARIES = [(k, k.split(".")[0], c) for k, c in _LAYER.items()]
HEAD_BOUNDARIES = [(k, k.split(".")[1], c) for k, c in _HEAD.items()]
MOE_ONLY = {"B8", "B9", "B10", "B11", "B12"}
STEP_INVARIANT_BOUNDARIES = ("B3.c_kv", "B3.k_pe", "B16.token")


def boundary_class(key):
    """The class of a boundary key, or None for any other key."""
    if key in _HEAD:
        return _HEAD[key]
    if not key.startswith("L") or "." not in key:
        return None
    suffix = key.split(".", 1)[1]
    if suffix.startswith("B11.expert_"):
        return _LAYER["B11.expert_*"]
    return _LAYER.get(suffix)


def boundary_id(key):
    return key.split(".")[1]


def boundary_iteration(key, iters):
    """Which decode iteration a dumped boundary of an `iters`-iteration run comes from: the
    cache rows at the handover position and the first token are written by iteration 0 only;
    every other workspace holds the last iteration's values."""
    if iters <= 1 or any(key.endswith(s) for s in STEP_INVARIANT_BOUNDARIES):
        return 0
    return iters - 1
