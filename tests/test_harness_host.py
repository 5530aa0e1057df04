"""The harness without a GPU:
* the reference's own driver calls work against this package: dry_run and build_plan with the
  positional arguments harness/run_fleet.py passes (:510-513), and every reference variant switch
  is accepted and recorded; refused options say why;
* harness/compare.py agrees with the reference's harness/compare.py (imported from the reference
  checkout when this container has it) on synthetic run directories: the same per-boundary metrics
  and verdicts, output-id and route-log results, growth curve and overall verdict."""
import importlib.util
import json
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "fleet-amd-task_b200" / "harness"
REF_HARNESS = Path("/root/reference/harness")


def test_reference_positional_dry_run_and_variants():
    from fleet import build_graph as B
    from fleet.pack_weights import REAL_DIMS
    # harness/run_fleet.py:510-513's positional call (debug_scores .. merge_oproj), then build_plan's
    plan, ops = B.dry_run(REAL_DIMS, 1056, 3, True, False, None, False, True, True, False, False, None, False, False,
                          True, 96, 400, True, True, 2, True, True)
    assert plan.variants["tile_linears"] and plan.variants["merge_halves"] == 2 and plan.variants["head_grid"] == 400
    assert plan.n_ops == len(ops) > 0
    plan, ops = B.dry_run(REAL_DIMS, 1056, 2, True, True, "L1.o_proj", True)   # debug, stop-after, debug_scores
    assert plan.calls[-1].label == "L1.o_proj" and "scores" in plan.tensors and "dbg_x_res_0" in plan.tensors
    assert any(c.method == "copy_layer" for c in plan.calls)
    with pytest.raises(ValueError):
        B.dry_run(REAL_DIMS, 1056, 2, True, False, None, False, False, False, False, False, "L1.qkva")
    with pytest.raises(ValueError):
        B.dry_run(REAL_DIMS, 1056, 2, True, merge_halves=2)   # halves need merge_tasks (the reference's rule)
    pj = B.plan_json(B.dry_run(REAL_DIMS, 1056, 2, True)[0])
    assert json.loads(json.dumps(pj))["variants"]["argmax_slices"] == 50


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.path.insert(0, str(Path(path).parent))
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.path.pop(0)
    return mod


def _synthetic_dirs(tmp):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(0)
    ref, fleet = {}, {}
    keys = ["L0.B1.norm1", "L0.B2.q", "L0.B3.c_kv", "L0.B6.attn", "L0.B7.x_res_attn", "L0.B13.layer_out",
            "L1.B8.router_logits", "L1.B12.shared", "head.B14.norm", "head.B15.logits"]
    for i, k in enumerate(keys):
        t = torch.randn(256, generator=g)
        ref[k] = t.to(torch.bfloat16)
        noise = (1e-3 if i % 3 else 4e-2) * torch.randn(256, generator=g)    # a few beyond their threshold
        fleet[k] = (t + noise).to(torch.bfloat16)
    ref["L1.B9.topk_idx"] = torch.tensor([3, 7, 1, 9, 4, 5], dtype=torch.int32)
    fleet["L1.B9.topk_idx"] = torch.tensor([7, 3, 1, 9, 4, 5], dtype=torch.int32)
    ref["L1.B10.topk_w"] = torch.tensor([0.3, 0.2, 0.1, 0.1, 0.05, 0.05])
    fleet["L1.B10.topk_w"] = torch.tensor([0.2, 0.3, 0.1, 0.1, 0.05, 0.05])
    ref["head.B16.token"] = torch.tensor([42])
    fleet["head.B16.token"] = torch.tensor([42])
    fleet["L5.B6.attn"] = fleet["L0.B6.attn"].clone()       # a layer the reference did not capture
    (tmp / "ref").mkdir()
    (tmp / "run").mkdir()
    save_file(ref, str(tmp / "ref" / "ref_boundaries_step0.safetensors"))
    save_file(fleet, str(tmp / "run" / "fleet_boundaries.safetensors"))
    (tmp / "ref" / "ref_output_ids.json").write_text(json.dumps([5, 6, 7, 8]))
    (tmp / "run" / "fleet_output_ids.json").write_text(json.dumps([5, 6, 9]))
    rl = [[{"idx": [1, 2, 3, 4, 5, 6], "w": [], "w_all": [0.1] * 8}], [{"idx": [1, 2, 3, 4, 5, 7], "w": [],
                                                                          "w_all": [0.1] * 8}]]
    (tmp / "ref" / "ref_route_log.json").write_text(json.dumps(rl))
    (tmp / "run" / "fleet_route_log.json").write_text(json.dumps([[{"idx": [1, 2, 3, 4, 5, 7, 64, 65], "w": []}],
                                                                  [{"idx": [1, 2, 3, 4, 5, 0], "w": []}]]))
    (tmp / "run" / "fleet_run_meta.json").write_text(json.dumps({"iters": 1, "head": True}))
    hid = torch.randn(4, 256, generator=g)
    save_file({"hidden": hid}, str(tmp / "ref" / "ref_hidden_per_layer_step0.safetensors"))
    save_file({"hidden": hid + 1e-3 * torch.randn(4, 256, generator=g)}, str(tmp / "run" / "fleet_hidden_per_layer.safetensors"))
    return tmp / "ref", tmp / "run"


@pytest.mark.skipif(not (REF_HARNESS / "compare.py").exists(), reason="the reference checkout is not in this container")
def test_compare_agrees_with_the_reference_compare(tmp_path):
    ref_dir, run_dir = _synthetic_dirs(tmp_path)
    ours = _load(HARNESS / "compare.py", "b200_compare")
    theirs = _load(REF_HARNESS / "compare.py", "reference_compare")
    a = ours.run(ref_dir, run_dir, None, tmp_path / "ours.md")
    b = theirs.run(ref_dir, run_dir, None, tmp_path / "theirs.md")
    assert [(r["key"], r["result"]) for r in a["boundaries"]] == [(r["key"], r["result"]) for r in b["boundaries"]]
    for ra, rb in zip(a["boundaries"], b["boundaries"]):
        for k in ("max_abs_err", "rel_err", "cos_sim"):
            if k in rb:
                assert ra[k] == pytest.approx(rb[k], rel=1e-12, abs=1e-15), (ra["key"], k)
    for k in ("output_ids", "route_log", "growth_curve"):
        assert a[k]["result"] == b[k]["result"], k
    assert a["output_ids"]["matched_prefix"] == b["output_ids"]["matched_prefix"]
    assert len(a["route_log"]["ties"]) == len(b["route_log"]["ties"])
    assert a["overall"] == b["overall"] == "FAIL"
    assert (a["n_pass"], a["n_fail"], a["n_not_captured"]) == (b["n_pass"], b["n_fail"], b["n_not_captured"])
