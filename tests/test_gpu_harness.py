"""The reference's run / compare flow against this package, on a B200: oracle/run_reference.py
writes the reference side for a 3-layer model of config 1 (seeded synthetic weights; the
reference writes the same files from its HF model), harness/run_fleet.py builds and runs the graph
through the reference-shaped surface (build() with the reference's arguments, compile(), one
launch) and dumps boundaries, ids and routes, and harness/compare.py must report PASS:
* one iteration with the per-layer snapshots: the head's boundaries and the cache rows of
  layers 0 and 1 at decode step 0, the growth curve;
* four iterations: the output ids, the route log and the boundaries against the reference's file
  for the last step;
* one iteration stopped after layer 1 (the reference's --stop-after): every boundary of layer 1
  (the workspaces hold the last writer's values, as in the reference's dumps)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
HARNESS = ROOT / "fleet-amd-task_b200" / "harness"


def _run(args, timeout=900):
    r = subprocess.run([sys.executable] + [str(a) for a in args], capture_output=True, text=True, timeout=timeout)
    return r.returncode, r.stdout[-4000:] + r.stderr[-4000:]


def test_run_fleet_and_compare_pass(tmp_path):
    ref = tmp_path / "ref"
    rc, log = _run([ROOT / "oracle" / "run_reference.py", "--out", ref, "--layers", 3, "--iters", 4])
    assert rc == 0, log
    for n, (iters, extra, min_compared) in enumerate(((1, ["--debug"], 5), (4, [], 5),
                                                      (1, ["--stop-after", "L1.combine"], 12))):
        out = tmp_path / f"fleet_{n}"
        rc, log = _run([HARNESS / "run_fleet.py", "--layers", 3, "--head", "--iters", iters, "--synthetic",
                        "--ref", ref, "--out", out, "--tile-linears", "--gemv-linears"] + extra)
        assert rc == 0, log
        for f in ("plan.json", "fleet_run_meta.json", "fleet_output_ids.json", "fleet_route_log.json",
                  "fleet_boundaries.safetensors", "wall.json"):
            assert (out / f).exists(), f
        rc, log = _run([HARNESS / "compare.py", "--ref", ref, "--fleet", out])
        assert rc == 0, log
        res = json.loads((out / "correctness_report.json").read_text())
        assert res["overall"] == "PASS" and res["n_fail"] == 0, res
        compared = [r for r in res["boundaries"] if r["result"] == "PASS"]
        assert len(compared) >= min_compared, [(r["key"], r["result"]) for r in res["boundaries"]]
        assert all(r.get("rel_err", 0.0) == 0.0 for r in compared), "the exact form must match bit for bit"
        if iters == 4:
            assert res["output_ids"]["result"] == "PASS" and res["route_log"]["result"] == "PASS"
        elif "--debug" in extra:
            assert res["growth_curve"]["result"] == "PASS"
        else:
            keys = {r["key"] for r in compared}
            assert {"L1.B2.q", "L1.B6.attn", "L1.B9.topk_idx", "L1.B12.shared", "L1.B13.layer_out"} <= keys, keys
