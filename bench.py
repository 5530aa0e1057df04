#!/usr/bin/env python3
"""Benchmark of the B200 decode megakernel: batch-1 greedy decode of the 27-layer
DeepSeek-V2-Lite-shaped model at 1K context, one persistent kernel launch per token.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

One step = one decode token (embedding, 27 layers, lm_head, argmax) = ONE launch of the
persistent kernel on the full model (seeded synthetic BF16 weights, 31.4 GB resident in HBM,
seeded synthetic latent cache of 1,023 prefilled rows). Every token reads ~4.9 GB of weights, far
more than the 126 MB L2, so no flush is needed between steps.

Prints one JSON line: metric ms/token (lower is better), the device-timed value, e2e through the
public API with host buffers (the input token copied H2D from pinned memory and the output token
D2H every step), the roofline of the kernel against the measured HBM copy bandwidth
(MEASURED_PEAKS.json), the CPU oracle's time for the same work on this host, the clocks seen.

`--impl reference` times the reference's CPU path (the oracle port of harness/numpy_ref.py
composed into the decode step, its row dots and attention in C on every host core; the
reference's own runtime is HIP for MI300X and its Fleet submodule is absent, so nothing else of it
can run here): W untimed and K timed whole decode tokens.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "fleet-amd-task_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "batch-1 decode ms/token (V2-Lite shape, 1K ctx); achieved HBM TB/s vs peak"
N_PROMPT = 1024
E2E_STEPS = 8


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c1", choices=["c1", "c0", "c2"],
                    help="c1: the decode step (the metric); c0: one MoE layer at position 1024; c2: the MLA "
                         "attention sweep (contexts 1K..32K, 8/16/32 splits); c0 and c2 print one line per case")
    ap.add_argument("--layers", type=int, default=27)
    ap.add_argument("--ctx", type=int, default=N_PROMPT,
                    help="prompt length (latent-cache rows + 1); 8192 is config 4's context (cache seed 5)")
    ap.add_argument("--cpu-sample-s", type=float, default=12.0, help="bound of the CPU baseline sample (s)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--routing", default="natural", choices=["natural", "uniform", "zipf"],
                    help="config 3's injected router logits (seed 4): uniform, or Zipf s=1.2 over the experts")
    ap.add_argument("--attend", default="exact", choices=["exact", "tc"],
                    help="MLA attention form: the bit-exact FP32 CUDA-core tasks, or the tensor-core tasks")
    ap.add_argument("--split", type=int, default=None, help="cache rows per attention split (default: the plan's)")
    ap.add_argument("--moe", default=None, choices=["units", "units_fp8", "staged"],
                    help="the experts' form (default: units on one GPU; expert parallelism is staged); "
                         "units_fp8: weight-only FP8 (E4M3) experts")
    ap.add_argument("--tc-parts", type=int, default=1, help="tensor-core attention: latent-column parts per split")
    ap.add_argument("--op-tasks", default="", help="task counts per operator kind, e.g. router=16,qkva=96")
    ap.add_argument("--trace", action="store_true",
                    help="record per-task %%globaltimer stamps and print a per-operator breakdown of the last "
                         "token to stderr (the timed numbers then include the stamping)")
    return ap.parse_args()


def peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML polled every 2 ms from
    a thread (a 16-token region lasts ~50 ms, shorter than nvidia-smi's start-up), else nvidia-smi
    every 200 ms. Read-only: no clock or setting is changed."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = {"sw_power_cap": "SwPowerCap", "hw_slowdown": "HwSlowdown", "sw_thermal_slowdown": "SwThermalSlowdown",
               "hw_thermal_slowdown": "HwThermalSlowdown"}

    def __init__(self, index, torch_device=None):
        self.index = index
        self.torch_device = torch_device
        self.proc = None
        self.lines = []
        self.samples = []         # (sm_mhz, reason bits) from NVML
        self.max_mhz = None
        self.nvml = None
        self._stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            pr = torch.cuda.get_device_properties(self.torch_device if self.torch_device is not None else 0)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        try:
            self.nvml, self.h = self._nvml_handle()
            self.max_mhz = float(self.nvml.nvmlDeviceGetMaxClockInfo(self.h, self.nvml.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _poll(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        while not self._stop.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)),
                                     int(get_reasons(self.h))))
            except Exception:
                pass
            time.sleep(0.002)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        self._stop.set()
        if self.nvml is not None:
            self.t.join(timeout=2)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        if self.nvml is not None:
            sm = [c for c, _ in self.samples]
            bits_of = {nm: getattr(self.nvml, f"nvmlClocksEventReason{k}", None) or
                       getattr(self.nvml, f"nvmlClocksThrottleReason{k}") for nm, k in self.REASONS.items()}
            reasons = sorted({nm for _, bits in self.samples for nm, b in bits_of.items() if bits & b})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(sm), "source": "nvml"}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


# ---------------------------------------------------------------------------------------------


def build_model(args, device, layers, ep=None):
    import torch
    from fleet import build_graph as B
    from fleet.workload import greedy_decode

    t0 = time.time()
    # config 1 (1K context): cache seed 1; config 4 (8K context): cache seed 5
    w = greedy_decode(device, n_prompt=args.ctx, new_tokens=args.warmup + args.steps + E2E_STEPS, layers=layers,
                      extra_rows=2)
    d, packed, capture, s_max, n_prompt = w.dims, w.packed, w.capture, w.s_max, w.n_prompt
    meta = B.make_meta(torch, s_max, w.prompt, n_prompt, device=device)
    routing = getattr(args, "routing", "natural")
    if routing != "natural":
        from fleet.capture import router_biases
        capture.update(router_biases(d, layers, routing, seed=4, device=device))
    extra = {} if args.split is None else dict(split=args.split)
    mpk, host, plan = B.build(packed, capture, meta, dims=d, s_max=s_max, layers=layers, head=True,
                              trace=args.trace, ep=ep, logit_bias=routing != "natural",
                              attend_tc=args.attend == "tc", tc_parts=args.tc_parts, op_tasks=op_tasks(args),
                              moe=args.moe, **extra)
    mpk.compile()
    torch.cuda.synchronize()
    build_model.workload = w
    return d, packed, capture, meta, mpk, host, plan, time.time() - t0


def op_tasks(args):
    """--op-tasks kind=n,... as a dict (None when empty)."""
    if not args.op_tasks:
        return None
    return {k: int(v) for k, v in (kv.split("=") for kv in args.op_tasks.split(","))}


def ids_check(meta, args, fp8=False):
    """The decoded tokens against the CPU oracle's 32 greedy ids of config 1
    (tests/golden/c1_greedy_ids.json): None when the workload is not config 1's. The FP8 experts
    decode other ids than the BF16 oracle's: their agreement is reported, not checked."""
    f = ROOT / "tests" / "golden" / "c1_greedy_ids.json"
    if not f.exists() or args.ctx != N_PROMPT or args.layers != 27 or args.routing != "natural":
        return None
    want = json.loads(f.read_text())["ids"]
    got = meta["tokens"][0, N_PROMPT:N_PROMPT + len(want)].tolist()
    n = min(len(want), args.warmup + args.steps + E2E_STEPS)
    if fp8:
        lead = next((i for i in range(n) if got[i] != want[i]), n)
        return {"ids_match": None, "compared": n, "fp8_equal_to_bf16_ids": sum(a == b for a, b in zip(got[:n], want)),
                "fp8_common_prefix": lead}
    return {"ids_match": got[:n] == want[:n], "compared": n}


def time_steps(mpk, meta, steps, torch, stream):
    """Device time of `steps` launches (one token each): events on the launching stream."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        starts[i].record(stream)
        mpk.launch(1, stream)
        ends[i].record(stream)
    torch.cuda.synchronize()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return per


def trace_summary(mpk, plan, out=sys.stderr):
    """Per-operator breakdown of the last launch's trace (one token): for each operator of a middle
    layer its task count, the most tasks one CTA ran, and the median task's prologue (activations
    loaded), stages (weights consumed), of which the consumers waited for a ring stage (wait), and
    epilogue (outputs, release); then, per operator kind,
    the median over the middle layers of how much it extends the token's critical path (its last
    task's end minus the latest end of every operator before it)."""
    import statistics as st
    recs = mpk.kernel.trace()
    labels = [c.label for c in plan.calls]
    by = {}
    for (op, task, cta, it, t_ready, t_end, t_body, t_stages, wait) in recs:
        by.setdefault(op, []).append((t_ready, t_end, t_body, t_stages, cta, wait))
    if not by:
        return
    ends = {op: max(r[1] for r in v) for op, v in by.items()}
    layers = sorted({int(lb[1:].split(".")[0]) for lb in labels if lb.startswith("L")})
    mid = layers[len(layers) // 2] if layers else None
    print(f"trace of one token: operators of layer {mid} (us; medians over tasks)", file=out)
    print("%-18s %6s %7s %8s %8s %8s %8s" % ("operator", "tasks", "max/cta", "prologue", "stages", "wait", "epilogue"),
          file=out)
    for op in sorted(by):
        if not labels[op].startswith(f"L{mid}."):
            continue
        v = by[op]
        per_cta = {}
        for r in v:
            per_cta[r[4]] = per_cta.get(r[4], 0) + 1
        pro = st.median([(r[2] - r[0]) / 1e3 for r in v if r[2]]) if any(r[2] for r in v) else 0.0
        stg = st.median([(r[3] - r[2]) / 1e3 for r in v if r[3] and r[2]]) if any(r[3] for r in v) else 0.0
        epi = st.median([(r[1] - (r[3] or r[2] or r[0])) / 1e3 for r in v])
        wt = st.median([r[5] / 1e3 for r in v])
        print("%-18s %6d %7d %8.2f %8.2f %8.2f %8.2f" % (labels[op], len(v), max(per_cta.values()), pro, stg, wt, epi),
              file=out)
    order = sorted(by)
    kinds = {}
    for i in range(1, len(order)):
        lab = labels[order[i]]
        if not lab.startswith("L"):
            continue
        l = int(lab[1:].split(".")[0])
        if l < 2 or l > layers[-1] - 1:
            continue
        prev = max(ends[o] for o in order[:i])
        kinds.setdefault(lab.split(".", 1)[1], []).append(max(0.0, (ends[order[i]] - prev) / 1e3))
    print("critical-path share per operator kind (us, median over the middle layers):", file=out)
    total = 0.0
    for k, v in kinds.items():
        total += st.median(v)
        print("  %-14s %7.2f" % (k, st.median(v)), file=out)
    t0 = min(r[0] for v in by.values() for r in v)
    print("  per layer      %7.2f; whole token %.1f" % (total, (max(ends.values()) - t0) / 1e3), file=out)


def time_e2e(mpk, meta, steps, torch, stream):
    """Through the public API with host buffers (mpk.decode_token, the library's mk_decode_token):
    per step the input token H2D from pinned memory, one launch, the output token D2H to pinned
    memory, and the wait for it on the host."""
    tok_in = torch.zeros(1, dtype=torch.int64, pin_memory=True)
    tok_out = torch.zeros(1, dtype=torch.int64, pin_memory=True)
    tokens = meta["tokens"]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    pos = mpk.step + 1
    tok_in.copy_(tokens[0, pos:pos + 1].cpu())
    e0.record(stream)
    t0 = time.perf_counter()
    for _ in range(steps):
        mpk.decode_token(tok_in, tok_out, stream)
        tok_in.copy_(tok_out)
    e1.record(stream)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) * 1e3 / steps
    return e0.elapsed_time(e1) / steps, wall


class CpuDecoder:
    """The CPU oracle decoding the same workload on this host: harness/numpy_ref.py's arithmetic
    (oracle/numpy_ref.py) composed into the decode step (oracle/model.py), its row dots and
    attention in C over the BF16 weights (oracle/detdot.c, one thread per host core unless
    ORACLE_THREADS says otherwise). The weights are copied to host memory once (31.4 GB at
    REAL_DIMS), outside any timing; each token is timed whole (embedding, every layer, head)."""

    def __init__(self, w, split):
        import numpy as np
        import torch
        from fleet.capture import softmax_scale
        from oracle import detmath
        from oracle.model import OracleModel

        def u16(t):
            return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)

        t0 = time.time()
        self.host = {k: u16(v) for k, v in w.packed.items()}
        d = w.dims
        self.model = OracleModel(d, self.host.__getitem__, lambda n, e: self.host[n][e],
                                 softmax_scale=softmax_scale(d.D_N, d.D_R), split=split)
        self.cache = {k: (u16(v).astype(np.uint32) << 16).view(np.float32) for k, v in w.capture.items()
                      if k.startswith(("c_kv_", "k_pe_"))}
        self.cos, self.sin = (w.capture[k].float().cpu().numpy() for k in ("cos", "sin"))
        self.tokens = np.zeros(w.s_max, np.int64)
        self.tokens[:w.n_prompt] = w.prompt
        self.pos = w.first_pos
        self.copy_s = time.time() - t0
        self.native = detmath._od() is not None
        self.threads = int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1)) if self.native else 1

    def token(self):
        """Decode one token; returns its wall time (s)."""
        t0 = time.perf_counter()
        tok, _, _ = self.model.step(int(self.tokens[self.pos]), self.pos, self.cache, self.cos, self.sin)
        dt = time.perf_counter() - t0
        self.tokens[self.pos + 1] = tok
        self.pos += 1
        return dt

    def describe(self, n):
        return (f"{n} whole decode tokens of the 27-layer model from position {self.pos - n} (every layer and the "
                f"head timed, nothing extrapolated); weights held as BF16 in host memory "
                f"(copied in {self.copy_s:.0f} s, not timed); {'C row dots and attention' if self.native else 'numpy'}"
                f" on {self.threads} thread(s) of {os.cpu_count()} host cores")


def cpu_baseline(w, split, budget_s):
    """A bounded sample of the same workload on the host cores: whole tokens until budget_s."""
    dec = CpuDecoder(w, split)
    times = []
    while not times or (sum(times) < budget_s and len(times) < 16):
        times.append(dec.token())
    v = sum(times) / len(times) * 1e3
    return {"value": round(v, 1), "unit": "ms/token", "cores": dec.threads, "kind": "port",
            "sample": dec.describe(len(times))}


def roofline(d, ms_per_token, ctx, bw_peak, peak_kind, world=1, expert_bytes=2, layers=None):
    """Algorithmic HBM bytes of one GPU's launch per token over its time: with expert parallelism
    rank 0 (the busiest) reads the replicated weights and the expert weights of ceil(N_SLOTS /
    world) of the eight slots. expert_bytes: 1 for the FP8 experts. layers: the graph's layers
    (the model's 27 by default); the committed traffic captures are of the 27-layer token."""
    from fleet.pack_weights import active_bytes_per_token, slot_bytes_per_token
    layers = d.L if layers is None else layers
    algo = active_bytes_per_token(d, ctx=ctx, layers=layers, expert_bytes=expert_bytes)
    if world > 1:
        mine = -(-d.N_SLOTS // world)
        algo -= slot_bytes_per_token(d, layers=layers) * (d.N_SLOTS - mine)
    achieved = algo / (ms_per_token * 1e-3) / 1e9
    traffic = None
    f = ROOT / "profiles" / ("decode_traffic.txt" if expert_bytes == 2 else "decode_traffic_fp8.txt")
    if f.exists() and world == 1 and layers == d.L:
        for line in f.read_text().splitlines():
            if line.startswith("traffic_bytes_per_token:"):
                traffic = float(line.split(":", 1)[1])
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": bw_peak, "unit": "GB/s",
            "frac": round(achieved / bw_peak, 4), "peak_kind": peak_kind, "traffic": traffic,
            "algorithmic_bytes": algo}


def run_ours(args):
    import torch

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = f"cuda:{local}"
    dist = None
    ep = None
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")     # no NVLink multicast objects in this job
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(device))
        from fleet.ep import EpGroup
        from fleet.pack_weights import REAL_DIMS as D

        def all_gather(obj):
            objs = [None] * ws
            dist.all_gather_object(objs, obj)
            return objs

        # expert parallelism by slot: rank r computes the slots s (six routed, two shared) with
        # s mod N = r; every rank holds every expert's weights and runs the rest of the graph
        ep = EpGroup(rank, ws, local, D.N_SLOTS, D.H, args.layers - 1, all_gather)
    d, packed, capture, meta, mpk, host, plan, t_setup = build_model(args, device, args.layers, ep)
    wl = build_model.workload
    stream = torch.cuda.Stream(device=device)
    mpk.step = args.ctx - 2
    for _ in range(args.warmup):
        mpk.launch(1, stream)
    torch.cuda.synchronize()
    st = mpk.status()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ctx0 = mpk.step + 2
    with ClockSampler(local, local) as clk:
        per = time_steps(mpk, meta, args.steps, torch, stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    st = mpk.status()
    ms = sum(per) / len(per)
    e2e_ms, e2e_wall = time_e2e(mpk, meta, E2E_STEPS, torch, stream)
    if args.trace and rank == 0:
        trace_summary(mpk, plan)
    st = mpk.status()
    ids = ids_check(meta, args, fp8=plan.moe == "units_fp8")
    if dist:
        # every rank must have decoded the same tokens and hold the same final residual
        n_dec = args.warmup + args.steps + E2E_STEPS
        mine = (meta["tokens"][0, args.ctx:args.ctx + n_dec].tolist(),
                int(host["x_res"].view(torch.int16).to(torch.int64).sum().item()), st["error"])
        every = all_gather(mine)
        ids = dict(ids or {}, ranks_agree=all(x == every[0] for x in every), ranks=ws)
        t = torch.tensor([ms, e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    bw, kind = peaks()
    ctx = ctx0 + args.steps // 2
    fp8 = plan.moe == "units_fp8"
    roof = roofline(d, ms, ctx, bw, kind, ws, expert_bytes=1 if fp8 else 2, layers=args.layers)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(wl, plan.split, args.cpu_sample_s)
        except MemoryError as e:            # the host could not hold the sample's weights
            cpu = {"value": None, "unit": "ms/token", "error": f"MemoryError: {e}"}
    if dist:
        dist.barrier()               # every peer is done writing into this rank's exchange buffers
        mpk.kernel.close()
        ep.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    out = {
        "metric": METRIC, "value": round(ms, 4), "unit": "ms/token", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16, e4m3 expert weights" if fp8 else "bf16",
        "data": f"synthetic: seeded BF16 weights N(0, 0.02), norms 1.0; seeded N(0,1) latent cache of "
                f"{args.ctx - 1:,} rows",
        "config": {"workload": ("C1: 27-layer DeepSeek-V2-Lite-shaped greedy decode, batch 1, 1 launch/token"
                                if args.ctx == N_PROMPT else
                                f"C4-shaped: the C1 model at {args.ctx}-token context, batch 1, 1 launch/token"),
                   "layers": args.layers, "ctx": [ctx0, ctx0 + args.steps - 1], "parallelism":
                   f"expert parallel x{ws}: the 8 expert slots (6 routed, 2 shared) dealt round-robin over the "
                   "GPUs, attention, router, layer 0 and head replicated; per-token latency is the max over ranks"
                   if ws > 1 else "1 GPU",
                   "l2": "no flush: 4.9 GB read per step >> 126 MB L2", "routing": args.routing,
                   "attention": ("tensor cores (mma.sync BF16, FP32 accumulation)" if args.attend == "tc" else
                                 "FP32 CUDA cores, specified summation order (bit-exact)"),
                   "split": plan.split, "moe": plan.moe, "tc_parts": args.tc_parts if args.attend == "tc" else None,
                   "op_tasks": op_tasks(args),
                   "tokens_per_s": round(1e3 / ms, 2)},
        "tokens_per_s": round(1e3 / ms, 2),
        "e2e": {"value": round(e2e_ms, 4), "unit": "ms/token", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8,
                "host_wall_ms": round(e2e_wall, 4)},
        "gpu_launches": args.steps,
        "roofline": roof,
        "cpu_baseline": cpu,
        "clocks": clk.summary(),
        "device_status": st["error_name"],
        "ids": ids,
        "setup_s": round(t_setup, 1),
        "ms_per_step_minmax": [round(min(per), 4), round(max(per), 4)],
    }
    print(json.dumps(out))


def run_reference(args):
    """The reference arm: the reference's CPU path for this workload (its NumPy arithmetic, restated
    by the oracle with the GEMVs and attention in C; the reference's own runtime is HIP for MI300X
    and cannot run here) on this host's cores, W untimed tokens then K timed ones, each a whole
    decode token. Rank 0 only."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    import torch
    from fleet import graph_plan as G
    from fleet.workload import greedy_decode
    device = "cuda:0" if torch.cuda.is_available() else "cpu"
    # the weights are the seeded synthetic ones of our arm (drawn by the CUDA generator on the GPU,
    # then copied to host memory once)
    w = greedy_decode(device, n_prompt=args.ctx, new_tokens=args.warmup + args.steps + 2, layers=args.layers)
    dec = CpuDecoder(w, args.split or G.SPLIT)
    del w
    torch.cuda.empty_cache()
    for _ in range(args.warmup):
        dec.token()
    times = [dec.token() for _ in range(args.steps)]
    v = sum(times) / len(times) * 1e3
    sample = dec.describe(args.steps)
    out = {"metric": METRIC, "value": round(v, 2), "unit": "ms/token", "n_gpus": ws, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(v, 2), "higher_is_better": False, "impl": "reference",
           "scaling": "strong", "vs_baseline": None,
           "dtype": "bf16 weights, FP32 accumulation (the reference's NumPy arithmetic; oracle port)",
           "data": "synthetic: the same seeded weights, cache and prompt as our arm",
           "config": {"workload": "C1: 27-layer DeepSeek-V2-Lite-shaped greedy decode, batch 1, on the host CPU",
                      "layers": args.layers, "ctx": [args.ctx + args.warmup, args.ctx + args.warmup + args.steps - 1]},
           "cpu_baseline": {"value": round(v, 2), "unit": "ms/token", "cores": dec.threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": round(v, 2), "unit": "ms/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "ms_per_step_minmax": [round(min(times) * 1e3, 1), round(max(times) * 1e3, 1)]}
    print(json.dumps(out))


# ---------------------------------------------------------------------------------------------
# config 0 and config 2: the operators of one layer, and the attention alone


def _flush_l2(torch, buf):
    buf.add_(1)            # 256 MiB written between timed launches: more than the 126 MB L2


def _time_kernel(torch, k, step, steps, warmup, before=None):
    """Device time (us) of single-iteration launches of handle k at position step + 1, L2 flushed
    between them; before(): per-launch input reset, outside the timed region."""
    flush = torch.zeros(64 << 20, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    times = []
    for i in range(warmup + steps):
        if before:
            before()
        _flush_l2(torch, flush)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        k.launch(1, step, s)
        e1.record(s)
        torch.cuda.synchronize()
        if i >= warmup:
            times.append(e0.elapsed_time(e1) * 1e3)
    assert k.status()["error"] == 0
    return times


def run_c2(args):
    """Config 2: the MLA decode attention (split-KV partials + merge + W_uv) alone, 16 heads of 576
    against one shared latent head, q and KV ~N(0,1) seed 3, at contexts 1K..32K with 8, 16 and 32
    splits, in both forms (the exact CUDA-core form where a split fits its ring, <= 168 rows)."""
    import torch
    from fleet import build_graph as B
    from fleet import mk
    from fleet.capture import softmax_scale
    from fleet.graph_plan import partials_row
    bw, kind = peaks()
    nh, d_r, d_c, d_v = 16, 64, 512, 128
    for ctx in (1024, 4096, 16384, 32768):
        g = torch.Generator(device="cuda").manual_seed(3)
        rn = lambda *sh: torch.randn(*sh, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
        ql, qp, ck, kp = rn(nh, d_c), rn(nh, d_r), rn(ctx, d_c), rn(ctx, d_r)
        W = (torch.randn(nh, d_v, d_c, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
        for n_splits in (8, 16, 32):
            split = -(-ctx // n_splits)
            for form in ("tc", "exact"):
                if form == "exact" and split > 168:
                    continue
                partials = torch.zeros((n_splits, nh, partials_row(d_c)), dtype=torch.float32, device="cuda")
                attn = torch.zeros(nh * d_v, dtype=torch.bfloat16, device="cuda")
                k = mk.MegaKernel(0)
                k.add(B.mla_attend_layer(mk, None, ql, qp, ck, kp, partials, softmax_scale(128, d_r), split, n_splits,
                                         nh if form == "tc" else 1, tc=form == "tc",
                                         col_parts=4 if form == "tc" and n_splits <= 16 else 1))
                k.add(B.mla_merge_uv_layer(mk, None, partials, W, attn, split, n_splits))
                k.finalize()
                t = _time_kernel(torch, k, ctx - 2, args.steps, args.warmup)
                k.close()
                us = sum(t) / len(t)
                algo = ctx * (d_c + d_r) * 2 + nh * (d_c + d_r) * 2 + nh * d_v * d_c * 2
                print(json.dumps({"metric": "MLA decode attention us/call (C2)", "value": round(us, 2), "unit": "us",
                                  "higher_is_better": False, "config": {"workload": "C2", "ctx": ctx,
                                  "n_splits": n_splits, "split_rows": split, "form": form},
                                  "steps": args.steps, "warmup": args.warmup, "l2": "flushed between launches",
                                  "roofline": {"bound": "hbm", "achieved": round(algo / us / 1e3, 1), "peak": bw,
                                               "unit": "GB/s", "frac": round(algo / us / 1e3 / bw, 4),
                                               "peak_kind": kind, "algorithmic_bytes": algo},
                                  "flops": 2 * nh * ctx * (d_c + d_r + d_c)}))


def run_c0(args):
    """Config 0: one MoE decoder layer (layer index 1) of the DeepSeek-V2-Lite shape at position 1024,
    seeded weights, hidden ~N(0,1), 1024 cached rows ~N(0,1) (seed 1): its nine operators in one
    launch, x_res restored before each (outside the timed region)."""
    import torch
    from fleet import build_graph as B
    from fleet import graph_plan as G
    from fleet.capture import make_capture
    from fleet.pack_weights import REAL_DIMS as d
    from fleet.pack_weights import moe_layer_bytes, synthetic_packed
    bw, kind = peaks()
    s_max, pos = 1056, 1024
    packed = synthetic_packed(d, layers=2, head=False, seed=0, device="cuda")
    capture = make_capture(d, 2, s_max, pos, seed=1, device="cuda")
    meta = B.make_meta(torch, s_max, [0] * (pos + 1), pos + 1)
    for form in ("exact", "tc"):
        plan = G.build_plan(d, s_max, 2, False, attend_tc=form == "tc")
        plan.calls = [c for c in plan.calls if c.label.startswith("L1.")]
        mpk, host, plan = B.build(packed, capture, meta, dims=d, s_max=s_max, layers=2, head=False, plan=plan)
        mpk.compile()
        x0 = torch.randn(d.H, generator=torch.Generator(device="cuda").manual_seed(7), device="cuda").to(torch.bfloat16)
        t = _time_kernel(torch, mpk.kernel, pos - 1, args.steps, args.warmup,
                         before=lambda: host["x_res"][0].copy_(x0))
        mpk.kernel.close()
        us = sum(t) / len(t)
        algo = moe_layer_bytes(d, ctx=pos + 1)
        print(json.dumps({"metric": "one MoE decoder layer us/step (C0)", "value": round(us, 2), "unit": "us",
                          "higher_is_better": False, "config": {"workload": "C0: layer 1 at position 1024",
                          "attention": form, "ops": plan.n_ops}, "steps": args.steps, "warmup": args.warmup,
                          "l2": "flushed between launches",
                          "roofline": {"bound": "hbm", "achieved": round(algo / us / 1e3, 1), "peak": bw, "unit": "GB/s",
                                       "frac": round(algo / us / 1e3 / bw, 4), "peak_kind": kind,
                                       "algorithmic_bytes": algo}}))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "c2":
        run_c2(args)
    elif args.config == "c0":
        run_c0(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
