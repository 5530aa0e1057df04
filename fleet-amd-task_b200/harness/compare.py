#!/usr/bin/env python3
"""Compare a run's dumped boundaries, ids and routes with a reference run and write the report.

    python harness/compare.py --ref REF_DIR --fleet RUN_DIR [--calibration FILE] [--report FILE]
    exit status 1 when a boundary or an exact check fails.

The reference's harness/compare.py (:36-236) is the contract: tensors are paired by boundary key
(harness/common.py), each is judged by rel_err = |a - b| / |b| (FP64 reductions over FP32 upcasts)
against its class threshold, B9 is compared as a set, B10 after aligning both sides by expert id,
B16 exactly; the output ids must match from the start (a shorter run passes as PARTIAL when every
id it made matches); a route mismatch is a tie (one expert swapped for one whose reference weight is
within tol of the larger), a cascade (after a tie) or a disagreement (the only kind that fails),
when the reference logged its 64 router weights, else any mismatch fails. Files read:

    REF_DIR:  ref_boundaries_step0.safetensors, ref_boundaries_step{K-1}.safetensors (optional),
              ref_output_ids.json, ref_route_log.json, ref_hidden_per_layer_step0.safetensors
    RUN_DIR:  fleet_boundaries.safetensors, fleet_output_ids.json, fleet_route_log.json,
              fleet_hidden_per_layer.safetensors (debug runs), fleet_run_meta.json
"""
import argparse
import json
import math
import re
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
import common  # noqa: E402

ROUTE_TOL_FALLBACK = 0.015      # tie band without a calibration (4 x the reference's router floor)


def metrics(a, b):
    """max_abs_err, rel_err (L2 of the difference over L2 of b) and cos_sim of a against b."""
    x = a.detach().cpu().double().flatten()
    y = b.detach().cpu().double().flatten()
    if x.numel() != y.numel():
        return {"shape_mismatch": [list(a.shape), list(b.shape)]}
    diff = x - y
    n_x, n_y = float(x.norm()), float(y.norm())
    mx = float(diff.abs().max()) if diff.numel() else 0.0
    if n_y > 0:
        rel = float(diff.norm()) / n_y
    else:
        rel = 0.0 if mx == 0 else math.inf
    if n_x > 0 and n_y > 0:
        cos = float(x @ y) / (n_x * n_y)
    else:
        cos = 1.0 if mx == 0 else 0.0
    return {"max_abs_err": mx, "rel_err": rel, "cos_sim": cos, "n": x.numel()}


def thresholds(calibration):
    th = dict(common.CLASS_THRESHOLD)
    if not calibration or "floor" not in calibration:
        return th, "starting values; not calibrated"
    for cls, floor in calibration["floor"].items():
        if cls in th and cls != "exact":
            th[cls] = common.THRESHOLD_MULTIPLIER * float(floor)
    return th, f"{common.THRESHOLD_MULTIPLIER:g} x calibrated floor"


def _layer(key):
    m = re.match(r"^L(\d+)\.", key)
    return int(m.group(1)) if m else None


def _order(key):
    l = _layer(key)
    if l is None:
        return (1 << 20, key)
    b = common.boundary_id(key)
    return (l, int(b[1:]) if b[1:].isdigit() else 99, key)


def _by_expert(key, fleet, ref):
    """B10 weights of both sides keyed by their B9 expert ids, in id order (the kernel lists the
    top-k by weight, the reference in its own order)."""
    k9 = key.replace(".B10.topk_w", ".B9.topk_idx")
    if k9 not in fleet or k9 not in ref:
        return fleet[key], ref[key], None
    f = {int(e): float(w) for e, w in zip(fleet[k9].flatten().tolist(), fleet[key].float().flatten().tolist())}
    r = {int(e): float(w) for e, w in zip(ref[k9].flatten().tolist(), ref[key].float().flatten().tolist())}
    if set(f) != set(r):
        return None, None, f"expert sets differ: fleet {sorted(f)} ref {sorted(r)}"
    ids = sorted(r)
    return torch.tensor([f[i] for i in ids]), torch.tensor([r[i] for i in ids]), None


def compare_boundaries(ref, fleet, th, floor=None, iters=1, ref_later=None):
    captured = sorted({_layer(k) for k in ref if _layer(k) is not None})
    rows = []
    for key in sorted(fleet, key=_order):
        cls = common.boundary_class(key)
        if cls is None:
            continue
        row = {"key": key, "boundary": common.boundary_id(key), "class": cls}
        rows.append(row)
        l = _layer(key)
        if l is not None and l not in captured:
            row.update(result="NOT_CAPTURED", detail=f"the reference captured layers {captured}")
            continue
        it = common.boundary_iteration(key, iters)
        side = ref
        if it > 0:
            row["iteration"] = it
            if ref_later is None:
                row.update(result="NOT_COMPARABLE", detail=f"dumped from iteration {it}, no reference for it")
                continue
            side = ref_later
        if key not in side:
            row["result"] = "MISSING_REF"
            continue
        a, b = fleet[key], side[key]
        if row["boundary"] == "B10":
            a, b, why = _by_expert(key, fleet, side)
            if why:
                row.update(result="FAIL", detail=why)
                continue
        if cls == "exact":
            if row["boundary"] == "B9":
                fa, fb = sorted(a.flatten().tolist()), sorted(b.flatten().tolist())
            else:
                fa, fb = int(a.flatten()[0]), int(b.flatten()[0])
            row.update(result="PASS" if fa == fb else "FAIL", detail=f"fleet {fa} ref {fb}")
            continue
        m = metrics(a, b)
        if "shape_mismatch" in m:
            row.update(result="FAIL", detail=f"shape mismatch {m['shape_mismatch']}")
            continue
        row.update(m, threshold=th[cls], floor=(floor or {}).get(cls))
        row["result"] = "PASS" if m["rel_err"] <= th[cls] else "FAIL"
    return rows


def compare_ids(ref_ids, fleet_ids):
    n = min(len(ref_ids), len(fleet_ids))
    first = next((i for i in range(n) if ref_ids[i] != fleet_ids[i]), None)
    if first is not None:
        result = "FAIL"
    else:
        result = "PASS" if len(fleet_ids) == len(ref_ids) else "PARTIAL"
    return {"n_ref": len(ref_ids), "n_fleet": len(fleet_ids), "compared": n,
            "matched_prefix": n if first is None else first, "first_divergence": first,
            "all_match": result == "PASS", "result": result}


def compare_route_log(ref_log, fleet_log, router_floor=None):
    with_weights = bool(ref_log) and all("w_all" in e for step in ref_log for e in step)
    tol = common.THRESHOLD_MULTIPLIER * float(router_floor) if router_floor else ROUTE_TOL_FALLBACK
    mism, ties, cascades, dis = [], [], [], []
    steps = min(len(ref_log), len(fleet_log))
    for s in range(steps):
        for j in range(min(len(ref_log[s]), len(fleet_log[s]))):
            r = sorted(ref_log[s][j]["idx"])
            f = sorted(fleet_log[s][j]["idx"][:len(r)])       # the run may log the forced experts too
            if r == f:
                continue
            m = {"step": s, "moe_layer_index": j, "ref": r, "fleet": f}
            mism.append(m)
            if not with_weights:
                continue
            gone, new = sorted(set(r) - set(f)), sorted(set(f) - set(r))
            if len(gone) == 1 and len(new) == 1:
                w = ref_log[s][j]["w_all"]
                wg, wn = float(w[gone[0]]), float(w[new[0]])
                m.update(left=gone[0], came=new[0], w_left=wg, w_came=wn, gap=abs(wg - wn), tol=tol * max(wg, wn))
                if m["gap"] <= m["tol"]:
                    m["class"] = "tie"
                    ties.append(m)
                    continue
            m["class"] = "cascade" if (ties or cascades) else "disagreement"
            (cascades if m["class"] == "cascade" else dis).append(m)
    if steps == 0:
        result = "SKIP"
    elif with_weights:
        result = "FAIL" if dis else "PASS"
    else:
        result = "FAIL" if mism else "PASS"
    return {"steps_compared": steps, "rule": "tie" if with_weights else "exact", "tol_rel": tol if with_weights else None,
            "mismatches": mism, "ties": ties, "cascades": cascades, "disagreements": dis, "result": result}


def growth_curve(ref_hidden, fleet_hidden, th_layer):
    n = min(ref_hidden.shape[0], fleet_hidden.shape[0])
    curve = [metrics(fleet_hidden[l], ref_hidden[l])["rel_err"] for l in range(n)]
    drops = [l for l in range(1, n) if curve[l] < 0.5 * curve[l - 1]]
    ok = bool(curve) and all(c <= th_layer for c in curve)
    return {"layers": n, "rel_err_per_layer": curve, "max_rel_err": max(curve) if curve else None,
            "within_threshold": ok, "note": f"drops by more than half at layers {drops}" if drops else "monotone",
            "result": ("PASS" if ok else "FAIL") if curve else "SKIP"}


def _fmt(x, nd=3):
    if x is None:
        return "-"
    if isinstance(x, float):
        return f"{x:.{nd}e}" if x != 0 and abs(x) < 1e-2 else f"{x:.{nd}f}"
    return str(x)


def write_report(path, res):
    out = ["# Correctness report", "", f"Thresholds: {res['threshold_source']}.", "",
           "| Key | Boundary | Class | max_abs_err | rel_err | cos_sim | floor | threshold | Result |",
           "|---|---|---|---|---|---|---|---|---|"]
    for r in res["boundaries"]:
        if "rel_err" in r:
            out.append(f"| `{r['key']}` | {r['boundary']} | {r['class']} | {_fmt(r['max_abs_err'])} | "
                       f"{_fmt(r['rel_err'])} | {_fmt(r['cos_sim'], 5)} | {_fmt(r['floor'])} | {_fmt(r['threshold'])} | "
                       f"**{r['result']}** |")
        else:
            out.append(f"| `{r['key']}` | {r['boundary']} | {r['class']} | - | - | - | - | exact | "
                       f"**{r['result']}** {r.get('detail', '')} |")
    out.append("")
    ids = res.get("output_ids")
    if ids:
        out.append(f"Output ids: **{ids['result']}**" + ("" if ids["result"] == "SKIP" else
                   f", {ids['matched_prefix']} of {ids['n_ref']} matched") + ".")
    rl = res.get("route_log")
    if rl:
        out.append(f"Route log: **{rl['result']}**" + ("" if rl["result"] == "SKIP" else
                   f", {rl['steps_compared']} steps, {len(rl['mismatches'])} mismatching (step, layer) pairs "
                   f"({rl['rule']} rule: {len(rl['ties'])} ties, {len(rl['cascades'])} cascades, "
                   f"{len(rl['disagreements'])} disagreements)") + ".")
    gc = res.get("growth_curve")
    if gc:
        out.append(f"Growth curve (B13 per layer): **{gc['result']}**, {gc['layers']} layers, max rel_err "
                   f"{_fmt(gc['max_rel_err'])}, {gc['note']}.")
    out += ["", f"Overall: **{res['overall']}** ({res['n_pass']} pass, {res['n_fail']} fail, {res['n_missing']} missing, "
                f"{res['n_not_comparable']} not comparable, {res['n_not_captured']} not captured)."]
    path.write_text("\n".join(out) + "\n")


def run(ref_dir, fleet_dir, calibration_path, report):
    from safetensors.torch import load_file
    ref_dir, fleet_dir, report = Path(ref_dir), Path(fleet_dir), Path(report)
    ref = load_file(str(ref_dir / "ref_boundaries_step0.safetensors"))
    fleet = load_file(str(fleet_dir / "fleet_boundaries.safetensors"))
    meta_f = fleet_dir / "fleet_run_meta.json"
    meta = json.loads(meta_f.read_text()) if meta_f.exists() else {}
    iters = int(meta.get("iters", 1) or 1)
    later_f = ref_dir / f"ref_boundaries_step{iters - 1}.safetensors"
    ref_later = load_file(str(later_f)) if iters > 1 and later_f.exists() else None
    cal = json.loads(Path(calibration_path).read_text()) if calibration_path and Path(calibration_path).exists() else None
    th, source = thresholds(cal)
    floor = cal.get("floor") if cal else None
    res = {"threshold_source": source, "thresholds": th, "iters": iters,
           "later_reference": later_f.name if ref_later is not None else None,
           "boundaries": compare_boundaries(ref, fleet, th, floor, iters, ref_later)}
    truncated = not meta.get("head", True) or bool(meta.get("stop_after"))
    ids_f = fleet_dir / "fleet_output_ids.json"
    if ids_f.exists():
        res["output_ids"] = ({"result": "SKIP", "note": "truncated graph: no head, ids are placeholders"} if truncated
                             else compare_ids(json.loads((ref_dir / "ref_output_ids.json").read_text()),
                                              json.loads(ids_f.read_text())))
    route_f = fleet_dir / "fleet_route_log.json"
    if route_f.exists():
        flog = json.loads(route_f.read_text())
        if any(any(e["idx"] for e in step) for step in flog) or not meta.get("stop_after"):
            res["route_log"] = compare_route_log(json.loads((ref_dir / "ref_route_log.json").read_text()), flog,
                                                 (floor or {}).get("router"))
        else:
            res["route_log"] = {"result": "SKIP", "note": "truncated graph: stopped before any router"}
    hid_f = fleet_dir / "fleet_hidden_per_layer.safetensors"
    if hid_f.exists():
        rh = load_file(str(ref_dir / "ref_hidden_per_layer_step0.safetensors"))["hidden"]
        res["growth_curve"] = growth_curve(rh, load_file(str(hid_f))["hidden"], th["layer"])
    verdicts = [r["result"] for r in res["boundaries"]]
    verdicts += [res[k]["result"] for k in ("output_ids", "route_log", "growth_curve")
                 if k in res and res[k]["result"] != "SKIP"]
    res.update(n_pass=verdicts.count("PASS") + verdicts.count("PARTIAL"), n_fail=verdicts.count("FAIL"),
               n_missing=verdicts.count("MISSING_REF"), n_not_comparable=verdicts.count("NOT_COMPARABLE"),
               n_not_captured=verdicts.count("NOT_CAPTURED"))
    res["overall"] = "PASS" if res["n_fail"] == 0 and res["n_missing"] == 0 and res["n_pass"] > 0 else "FAIL"
    report.parent.mkdir(parents=True, exist_ok=True)
    write_report(report, res)
    report.with_suffix(".json").write_text(json.dumps(res, indent=2) + "\n")
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True)
    ap.add_argument("--fleet", required=True)
    ap.add_argument("--calibration", default=None, help="default: <ref>/calibration.json if present")
    ap.add_argument("--report", default=None, help="default: <fleet>/correctness_report.md")
    a = ap.parse_args()
    cal = a.calibration or str(Path(a.ref) / "calibration.json")
    report = a.report or str(Path(a.fleet) / "correctness_report.md")
    res = run(a.ref, a.fleet, cal, report)
    for r in res["boundaries"]:
        tail = f" rel_err {_fmt(r.get('rel_err'))} thr {_fmt(r.get('threshold'))}" if "rel_err" in r else f" {r.get('detail', '')}"
        print(f"{r['result']:14s} {r['key']:28s}{tail}")
    for k in ("output_ids", "route_log", "growth_curve"):
        if k in res:
            print(f"{res[k]['result']:14s} {k}")
    print(f"overall: {res['overall']}  -> {report}")
    sys.exit(0 if res["overall"] == "PASS" else 1)


if __name__ == "__main__":
    main()
