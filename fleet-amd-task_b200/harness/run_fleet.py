#!/usr/bin/env python3
"""Build and run the B200 decode graph, then dump what compare.py reads.

    python harness/run_fleet.py --layers N [--head] [--iters K] [--debug] [--debug-scores]
        [--stop-after L1.o_proj] (--model-dir SNAPSHOT | --synthetic) [--ref REF_DIR] [--out DIR]
        [--split N] [--attend-tc] [--moe units|units_fp8|staged] [--event-timing] [--align-alloc BYTES] [--workspaces-first]
        [the reference's variant switches: --tile-linears ... --merge-oproj, recorded]

The driver of the reference (harness/run_fleet.py:505-616), against this package: positions follow
its D14/D15 (step = n_prompt - 2, the first iteration at n_prompt - 1, every iteration in one
launch), the capture comes from the reference side's REF_DIR/ref_cache.safetensors (cos, sin and the
prefill's latent cache [L, S, 512] / [L, S, 64]) and the prompt from REF_DIR/prompt_ids.json, and the
same files come out:

    plan.json, fleet_run_meta.json, wall.json, fleet_output_ids.json, fleet_route_log.json,
    fleet_boundaries.safetensors, fleet_hidden_per_layer.safetensors (--debug)

--model-dir packs a real checkpoint (fleet.pack_weights.pack_all); --synthetic draws the benchmark
configs' seeded weights (fleet.workload). Boundaries other than the cache rows and the first token
hold the last iteration's values (harness/common.py boundary_iteration).
"""
import argparse
import json
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent))
import common  # noqa: E402

VARIANT_FLAGS = ("tile_linears", "attend_tasks", "fuse_norm2", "fuse_silu", "fuse_norm1", "prefetch", "gemv_linears",
                 "gemv_w13", "merge_tasks", "router_tasks", "merge_oproj")


def writers(calls, output_args):
    """tensor name -> label of the last operator that wrote it, in plan order."""
    w = {}
    for c in calls:
        for k in output_args[c["method"]]:
            v = c["args"].get(k)
            if v is None:
                continue
            for name in (v if isinstance(v, list) else [v]):
                w[name["tensor"] if isinstance(name, dict) else name] = c["label"]
    return w


def boundary_dump(plan, host, tokens, n_prompt, dims, iters=1):
    """Map the workspaces to boundary keys from who wrote each last. plan: plan_json(); host: name ->
    tensor. The B200 graph fuses the norms into their GEMVs, so `h` is written by L{l}.qkva (norm1),
    L0.gate_up or L{l}.router (norm2) and head.lm_head (the final norm). Returns (dict, notes)."""
    from fleet.graph_plan import OUTPUT_ARGS
    w = writers(plan["calls"], OUTPUT_ARGS)
    b, notes = {}, []
    if iters != 1:
        notes.append(f"boundaries other than {', '.join(common.STEP_INVARIANT_BOUNDARIES)} are from iteration "
                     f"{iters - 1}")

    def put(key, t):
        b[key] = t.detach().cpu().contiguous().clone()

    def layer(label):
        return int(label.split(".")[0][1:])

    lab = w.get("h")
    if lab:
        if lab.endswith(".qkva"):
            put(f"L{layer(lab)}.B1.norm1", host["h"][0])
        elif lab.endswith((".router", ".gate_up")):
            put(f"L{layer(lab)}.norm2", host["h"][0])
        elif lab == "head.lm_head":
            put("head.B14.norm", host["h"][0])
    lab = w.get("qkva")
    if lab:
        put(f"L{layer(lab)}.B2.q", host["qkva"][0, :dims.Q_OUT])
        put(f"L{layer(lab)}.kva", host["qkva"][0, dims.Q_OUT:])
    lab = w.get("q_pe")
    if lab:
        put(f"L{layer(lab)}.B4.q_pe", host["q_pe"])
        put(f"L{layer(lab)}.ql_nope", host["ql_nope"])
    for name in w:
        if name.startswith("c_kv_"):
            l = int(name.split("_")[-1])
            put(f"L{l}.B3.c_kv", host[name][n_prompt - 1])
            put(f"L{l}.B3.k_pe", host[f"k_pe_{l}"][n_prompt - 1])
    lab = w.get("scores")
    if lab:
        put(f"L{layer(lab)}.B5.scores", host["scores"][:, :n_prompt])
    lab = w.get("attn")
    if lab:
        put(f"L{layer(lab)}.B6.attn", host["attn"][0])
    lab = w.get("x_res")
    if lab:
        if lab.endswith(".o_proj"):
            put(f"L{layer(lab)}.B7.x_res_attn", host["x_res"][0])
        elif lab.endswith((".w2_combine", ".combine", ".down")):
            put(f"L{layer(lab)}.B13.layer_out", host["x_res"][0])
        elif lab == "prologue.embed":
            put("prologue.embed", host["x_res"][0])
    lab = w.get("mask")
    if lab:
        l, k = layer(lab), dims.TOPK
        mask = host["mask"].cpu()
        put(f"L{l}.B8.router_logits", host["logits_router"][0])
        put(f"L{l}.B9.topk_idx", mask[:k])
        put(f"L{l}.B10.topk_w", host["topk_w"][0, :k])
        if w.get("out8") and layer(w["out8"]) == l:
            out8 = host["out8"]
            for s in range(k):
                put(f"L{l}.B11.expert_{int(mask[s])}", out8[s])
            put(f"L{l}.B12.shared", sum(out8[s].float() for s in range(k, dims.N_SLOTS)))
    if w.get("logits"):
        put("head.B15.logits", host["logits"][0])
    if w.get("tokens"):
        put("head.B16.token", tokens[0, n_prompt:n_prompt + 1])
    hidden = [host[f"dbg_x_res_{l}"][0] for l in range(plan["layers"]) if f"dbg_x_res_{l}" in w]
    if hidden:
        import torch
        b["_hidden"] = torch.stack([h.detach().cpu() for h in hidden])
    return b, notes


def build_parser():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, required=True)
    ap.add_argument("--head", action="store_true")
    ap.add_argument("--iters", type=int, default=1)
    ap.add_argument("--debug", action="store_true", help="per-layer residual snapshots (growth curve)")
    ap.add_argument("--debug-scores", action="store_true", help="dump the attention scores (boundary B5)")
    ap.add_argument("--stop-after", default=None, help="operator label, e.g. L1.o_proj")
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--model-dir", default=None, help="a checkpoint snapshot (config.json + safetensors)")
    src.add_argument("--synthetic", action="store_true", help="the benchmark configs' seeded synthetic weights")
    ap.add_argument("--ref", required=True, help="the reference side's directory (ref_cache, prompt_ids.json)")
    ap.add_argument("--prompt", default=None, help="default: <ref>/prompt_ids.json")
    ap.add_argument("--out", required=True)
    ap.add_argument("--split", type=int, default=None, help="cache rows per attention split")
    ap.add_argument("--attend-tc", action="store_true", help="the MLA attention on the tensor cores")
    ap.add_argument("--moe", default=None, choices=["units", "units_fp8", "staged"],
                    help="the experts' form (default: units; units_fp8: weight-only FP8 experts)")
    ap.add_argument("--event-timing", action="store_true", help="per-task %%globaltimer stamps (event_timing.json)")
    ap.add_argument("--align-alloc", type=int, default=0, help="re-base weights, capture and workspaces on BYTES")
    ap.add_argument("--workspaces-first", action="store_true", help="allocate the workspaces before the weights")
    for f in VARIANT_FLAGS:
        ap.add_argument("--" + f.replace("_", "-"), action="store_true", help="reference graph variant (recorded)")
    ap.add_argument("--linear-grid", type=int, default=None)
    ap.add_argument("--head-grid", type=int, default=None)
    ap.add_argument("--merge-halves", type=int, default=1)
    return ap


def main(argv=None):
    args = build_parser().parse_args(argv)
    import torch
    from safetensors.torch import load_file, save_file

    from fleet import build_graph as B
    from fleet import graph_plan as G
    from fleet.pack_weights import REAL_DIMS, Dims, pack_all, synthetic_packed

    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    ref_dir = Path(args.ref)
    prompt = json.loads(Path(args.prompt or ref_dir / "prompt_ids.json").read_text())
    n_prompt = len(prompt)
    s_max = n_prompt + args.iters
    dims = (Dims.from_config(json.loads((Path(args.model_dir) / "config.json").read_text())) if args.model_dir
            else REAL_DIMS)
    variants = {f: getattr(args, f) for f in VARIANT_FLAGS}
    variants.update(linear_grid=args.linear_grid, head_grid=args.head_grid, merge_halves=args.merge_halves)
    kw = {} if args.split is None else dict(split=args.split)
    kw["moe"] = args.moe
    # the plan's checks run on the dry run, before any weight is packed (the reference's order)
    B.dry_run(dims, s_max, args.layers, args.head, args.debug, args.stop_after, args.debug_scores,
              args.tile_linears, args.attend_tasks, args.fuse_norm2, args.fuse_silu, None, args.fuse_norm1,
              args.prefetch, args.gemv_linears, args.linear_grid, args.head_grid, args.gemv_w13, args.merge_tasks,
              args.merge_halves, args.router_tasks, args.merge_oproj, attend_tc=args.attend_tc, **kw)
    t0 = time.time()
    workspaces = None
    if args.workspaces_first:
        pre = G.build_plan(dims, s_max, args.layers, args.head, args.debug, args.debug_scores, attend_tc=args.attend_tc,
                           **kw)
        workspaces = B.allocate_workspaces(torch, pre, args.align_alloc)
    if args.model_dir:
        packed = pack_all(args.model_dir, "cuda", dims, layers=args.layers, head=args.head or None)
    else:
        packed = synthetic_packed(dims, layers=args.layers, head=args.head, seed=0, device="cuda")
    if args.align_alloc:
        packed = {k: B.aligned_copy(torch, v, args.align_alloc) for k, v in packed.items()}
    t_pack = time.time() - t0
    cache = load_file(str(ref_dir / "ref_cache.safetensors"))
    capture = {"cos": cache["cos"][:s_max].contiguous().cuda(), "sin": cache["sin"][:s_max].contiguous().cuda()}
    for l in range(args.layers):
        capture[f"c_kv_{l}"] = cache["c_kv"][l, :s_max].contiguous().cuda()
        capture[f"k_pe_{l}"] = cache["k_pe"][l, :s_max].contiguous().cuda()
    if args.align_alloc:
        capture = {k: B.aligned_copy(torch, v, args.align_alloc) for k, v in capture.items()}
    meta = B.make_meta(torch, s_max, prompt, n_prompt)
    t1 = time.time()
    mpk, host, plan = B.build(packed, capture, meta, dims, s_max, args.layers, args.head, args.debug, args.stop_after,
                              args.debug_scores, align=args.align_alloc, workspaces=workspaces,
                              trace=args.event_timing, attend_tc=args.attend_tc, **variants, **kw)
    pj = B.plan_json(plan)
    (out / "plan.json").write_text(json.dumps(pj) + "\n")
    mpk.compile(output_dir=str(out / "build"))
    t_build = time.time() - t1
    meta["step"].fill_(n_prompt - 2)
    meta["tokens"][0, n_prompt:] = 0
    torch.cuda.synchronize()
    run_meta = {"layers": args.layers, "head": args.head, "iters": args.iters, "debug": args.debug,
                "debug_scores": args.debug_scores, "stop_after": args.stop_after, "s_max": s_max,
                "n_prompt": n_prompt, "attend_tc": args.attend_tc, "split": plan.split, "variants": plan.variants,
                "ops": len(pj["calls"]), "tasks": sum(c["tasks"] for c in pj["calls"]),
                "weights": args.model_dir or "synthetic (seed 0)", "align_alloc": args.align_alloc,
                "workspaces_first": args.workspaces_first, "completed": False}
    (out / "fleet_run_meta.json").write_text(json.dumps(run_meta, indent=2) + "\n")
    t2 = time.time()
    mpk()
    torch.cuda.synchronize()
    t_run = time.time() - t2
    status = mpk.status(raise_on_error=False)
    if args.event_timing:
        recs = mpk.kernel.trace()
        labels = [c["label"] for c in pj["calls"]]
        (out / "event_timing.json").write_text(json.dumps(
            [{"op": labels[r[0]], "task": r[1], "cta": r[2], "iter": r[3], "ready_ns": r[4], "end_ns": r[5]}
             for r in recs]) + "\n")
    ids = meta["tokens"][0, n_prompt:n_prompt + args.iters].cpu().tolist()
    (out / "fleet_output_ids.json").write_text(json.dumps(ids) + "\n")
    b, notes = boundary_dump(pj, host, meta["tokens"], n_prompt, dims, args.iters)
    hidden = b.pop("_hidden", None)
    save_file({k: v.contiguous() for k, v in b.items()}, str(out / "fleet_boundaries.safetensors"))
    if hidden is not None:
        save_file({"hidden": hidden.contiguous()}, str(out / "fleet_hidden_per_layer.safetensors"))
    if "route_log" in host:
        rl = host["route_log"].cpu()
        # the MoE layers whose router is in the plan (a --stop-after plan ends before the rest)
        n_moe = sum(1 for c in pj["calls"] if c["label"].endswith(".router"))
        log = [[{"idx": rl[s % rl.shape[0], j].tolist(), "w": []} for j in range(n_moe)] for s in range(args.iters)]
        (out / "fleet_route_log.json").write_text(json.dumps(log) + "\n")
    wall = {"mpk_wall_s": t_run, "iters": args.iters, "pack_s": t_pack, "build_s": t_build}
    (out / "wall.json").write_text(json.dumps(wall) + "\n")
    run_meta.update(boundary_keys=sorted(b), output_ids=ids, notes=notes, timings_s=wall,
                    device_status=status["error_name"], completed=status["error"] == 0)
    (out / "fleet_run_meta.json").write_text(json.dumps(run_meta, indent=2) + "\n")
    mpk.kernel.close()
    print(f"ids {ids}; {len(b)} boundary tensors; status {status['error_name']}; one launch of {args.iters} "
          f"iterations {t_run * 1e3:.1f} ms -> {out}")
    return 0 if status["error"] == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
