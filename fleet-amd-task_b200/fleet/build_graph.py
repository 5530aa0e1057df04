#!/usr/bin/env python3
"""Build the B200 persistent decode kernel from a plan (drop-in for the reference's
fleet/build_graph.py: build(), make_meta(), plan_json(), dry_run(), the layer methods).

    mpk, host, plan = build(packed, capture, meta, dims=..., s_max=..., layers=N, head=True)
    mpk.compile(output_dir=...)       # builds and uploads the schedule (no code generation)
    mpk()                              # one launch: every remaining greedy iteration

Each plan call becomes one operator of the C library (include/fleet_mk.h) through ctypes; torch
only allocates the workspaces and hands their device pointers over. `dry_run` drives the same
code against a recorder, so the plan's checks run without a GPU.
"""
import argparse
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from fleet import graph_plan as G  # noqa: E402
from fleet.pack_weights import Dims, REAL_DIMS  # noqa: E402

TORCH_DTYPES = {"bf16": "bfloat16", "f32": "float32", "i32": "int32", "i64": "int64", "u8": "uint8"}


# ----------------------------------------------------------------------------
# the layer methods: plan call -> MkOp


def embed_layer(mk, t, input, weight, output):
    return mk.make_op(mk.OP_EMBED, 0, {0: weight, 1: input, 2: output}, {0: weight.shape[0], 1: weight.shape[1]})


def linear_gemv_layer(mk, t, input, weight, output, w_norm=None, residual=None, h_out=None, tokens_out=None,
                      norm=False, residual_add=False, argmax=False, eps=G.RMS_EPS):
    N, K = weight.shape
    assert input.numel() == K and output.numel() == N, (input.shape, weight.shape, output.shape)
    flags = (mk.F_NORM if norm else 0) | (mk.F_RESIDUAL if residual_add else 0) | (mk.F_ARGMAX if argmax else 0)
    g = mk.P["gemv"]
    return mk.make_op(mk.OP_GEMV, flags, {g["X"]: input, g["WNORM"]: w_norm, g["W"]: weight, g["RES"]: residual,
                                          g["OUT"]: output, g["HOUT"]: h_out, g["TOKENS"]: tokens_out},
                      {0: N, 1: K}, {0: eps})


def mla_prep_layer(mk, t, qkva, w_kv_norm, w_ukT, cos, sin, c_kv, k_pe, ql_nope, q_pe, eps=G.RMS_EPS):
    nh, d_c, d_n = w_ukT.shape
    d_r = k_pe.shape[1]
    assert qkva.numel() == nh * (d_n + d_r) + d_c + d_r
    return mk.make_op(mk.OP_MLA_PREP, 0, dict(enumerate([qkva, w_kv_norm, w_ukT, cos, sin, c_kv, k_pe, ql_nope, q_pe])),
                      {0: nh, 1: d_n, 2: d_r, 3: d_c, 4: c_kv.shape[0]}, {0: eps})


def mla_attend_layer(mk, t, ql_nope, q_pe, c_kv, k_pe, partials, softmax_scale, split, n_splits, head_group,
                     tc=False, scores=None, col_parts=1):
    """tc: the tensor-core form (one task per split for all heads; head_group must be the head
    count), else the FP32 CUDA-core form in the specified summation orders (bit-exact).
    scores: optional [nh, s_max] FP32 output of the scaled scores (the reference's debug_scores,
    boundary B5). col_parts (tc): latent-column parts per split, one task each (1, 2, 4 or 8)."""
    nh, d_c = ql_nope.shape
    assert partials.shape == (n_splits, nh, G.partials_row(d_c)), partials.shape
    assert not tc or head_group == nh, "the tensor-core attention takes all heads of a split in one task"
    assert scores is None or tuple(scores.shape) == (nh, c_kv.shape[0]), "scores: [heads, s_max]"
    return mk.make_op(mk.OP_MLA_ATTEND, mk.F_TC if tc else 0,
                      dict(enumerate([ql_nope, q_pe, c_kv, k_pe, partials, scores])),
                      {0: nh, 1: d_c, 2: k_pe.shape[1], 3: c_kv.shape[0], 4: split, 5: head_group, 6: n_splits,
                       7: partials.shape[2], 8: col_parts}, {0: softmax_scale})


def mla_merge_uv_layer(mk, t, partials, w_uv, output, split, n_splits):
    nh, d_v, d_c = w_uv.shape
    return mk.make_op(mk.OP_MLA_MERGE_UV, 0, {0: partials, 1: w_uv, 2: output},
                      {0: nh, 1: d_v, 2: d_c, 3: split, 4: n_splits, 5: partials.shape[2]})


def moe_router_layer(mk, t, input, w_norm, w_gate, h, topk_w, routing, mask, logits, route_log, layer_index, topk,
                     n_experts, n_forced, scaling, eps, bias=None, logit_tag=None, mask_tag=None):
    """logit_tag [E] / mask_tag [TOPK + n_forced] int64: the tagged-word hand-offs (fleet_mk.h
    MK_P_RT_LOGTAG, MK_P_RT_MASKTAG): task 0 routes from the tasks' tagged logits, and the expert
    units read the slots' experts from the tagged words without waiting for the router."""
    E, H = w_gate.shape
    r = mk.P["rt"]
    log_rows, log_layers, log_slots = route_log.shape if route_log is not None else (1, 1, topk + n_forced)
    return mk.make_op(mk.OP_ROUTER, 0, {r["X"]: input, r["WNORM"]: w_norm, r["WGATE"]: w_gate, r["HOUT"]: h,
                                        r["LOGITS"]: logits, r["TOPKW"]: topk_w, r["ROUTING"]: routing,
                                        r["MASK"]: mask, r["ROUTELOG"]: route_log, r["BIAS"]: bias,
                                        r["LOGTAG"]: logit_tag, r["MASKTAG"]: mask_tag},
                      {0: H, 1: E, 2: topk, 3: n_forced, 4: layer_index, 5: log_layers * log_slots, 6: log_rows},
                      {0: eps, 1: scaling})


def gateup_layer(mk, t, input, weight, act, inter, groups, expert, norm, w_norm=None, mask=None, mid=None, h_out=None,
                 eps=G.RMS_EPS, static_ids=False, ep=None):
    """static_ids: the mask holds constant expert ids (the shared experts), so the weights stream
    without waiting for a router. ep (rank, world, slot0): expert parallelism by slot, only the
    groups g whose slot slot0 + g has (slot0 + g) mod world = rank, spread over the tasks."""
    K = weight.shape[-1]
    estride = weight.shape[-2] * K if weight.dim() == 3 else 0
    nexp = weight.shape[0] if weight.dim() == 3 else 1
    flags = (mk.F_EXPERT if expert else 0) | (mk.F_NORM if norm else 0) | (mk.F_STATIC_IDS if static_ids else 0)
    ips = {0: K, 1: inter, 2: groups, 3: estride, 4: nexp}
    if ep is not None:
        flags |= mk.F_EP
        ips.update({5: ep[0], 6: ep[1], 7: ep[2] if len(ep) > 2 else 0})
    u = mk.P["gu"]
    return mk.make_op(mk.OP_GATEUP, flags, {u["X"]: input, u["WNORM"]: w_norm, u["W"]: weight, u["MASK"]: mask,
                                            u["MID"]: mid, u["ACT"]: act, u["HOUT"]: h_out}, ips, {0: eps})


def moe_w2_combine_layer(mk, t, input, weight, mask, topk_w, residual, output, out8=None, ep=None, peers=None,
                         topk=None, layer=0):
    """ep (rank, world): expert parallelism by slot; the task computes its rank's slots (s mod world
    = rank) for its rows, exchanges them with the same task of every peer (`peers`, fleet/ep.py)
    and combines all slots (out8 is then not written)."""
    E, H, I = weight.shape
    assert residual.data_ptr() == output.data_ptr(), "the combine adds into x_res in place"
    n_slots = input.shape[0]
    w = mk.P["w2"]
    flags, ips = 0, {0: H, 1: I, 2: n_slots, 3: H * I, 4: E}
    if ep is not None:
        flags = mk.F_EP
        ips.update({5: topk, 6: ep[0], 7: ep[1], 8: layer})
    return mk.make_op(mk.OP_W2_COMBINE, flags, {w["ACT"]: input, w["W"]: weight, w["MASK"]: mask, w["TOPKW"]: topk_w,
                                                w["XRES"]: output, w["OUT8"]: out8, w["PEERS"]: peers}, ips)





def moe_units_layer(mk, t, input, w13, w2f, sums, slot0, nslots, inter, w_norm=None, mask=None, act=None,
                    h_out=None, norm=False, fixed0=None, static_experts=None, mask_tag=None, scale13=None,
                    eps=G.RMS_EPS):
    """Expert units of slots [slot0, slot0 + nslots): gate/up + SwiGLU of each unit's intermediates
    and the down projection's butterfly subtree sums into `sums` [NS, parts, 8, H]. w13 [E, 2I, H]
    (gate/up interleaved), w2f the down projection regrouped by unit (pack_weights.regroup_w2).
    Slots from fixed0 on use experts static_experts, static_experts + 1, ... (the shared experts,
    no router); the slots before fixed0 take theirs from `mask` once the router is done. Every
    task runs a share of the fixed slots' units, then a share of the routed slots'. mask_tag: the
    router's tagged slot experts (the routed weights stream as soon as those words are in).
    scale13 [E, 2] FP32: FP8 experts (fleet_mk.h MK_F_FP8), w13 and w2f then hold E4M3 codes
    (pack_weights.fp8_experts) and scale13 the gate and up scales."""
    E, two_i, H = w13.shape
    assert two_i == 2 * inter and w2f.shape == (E, H * inter), (tuple(w13.shape), tuple(w2f.shape))
    ns = sums.shape[0]
    fixed0 = slot0 + nslots if fixed0 is None else fixed0
    assert slot0 <= fixed0 <= slot0 + nslots and (fixed0 == slot0 + nslots or static_experts is not None)
    flags = (mk.F_NORM if norm else 0) | (mk.F_EXPERT if fixed0 > slot0 else 0) | (mk.F_FP8 if scale13 is not None
                                                                                     else 0)
    assert scale13 is None or tuple(scale13.shape) == (E, 2), tuple(scale13.shape)
    ips = {0: H, 1: inter, 2: slot0, 3: nslots, 4: ns, 5: E, 7: fixed0}
    if fixed0 < slot0 + nslots:
        flags |= mk.F_STATIC_IDS
        ips[6] = static_experts
    u = mk.P["mu"]
    return mk.make_op(mk.OP_MOE_UNITS, flags, {u["X"]: input, u["WNORM"]: w_norm, u["W13"]: w13, u["W2F"]: w2f,
                                               u["MASK"]: mask, u["SUMS"]: sums, u["ACT"]: act, u["HOUT"]: h_out,
                                               u["MASKTAG"]: mask_tag, u["SCALE13"]: scale13},
                      ips, {0: eps})


def moe_combine_layer(mk, t, sums, topk_w, residual, output, inter, out8=None, mask=None, scale2=None):
    """out8 = bf16(down projection) per slot from the units' subtree sums, then
    x_res = bf16(x_res + sum_s f32(out8_s w_s)) (numpy_ref.moe_combine), in place. scale2 [E] FP32:
    FP8 experts, each slot's down projection times its expert's (mask[s]) scale before the rounding."""
    assert residual.data_ptr() == output.data_ptr(), "the combine adds into x_res in place"
    assert scale2 is None or mask is not None, "FP8 down scales need the slots' experts"
    ns, H = sums.shape[0], sums.shape[-1]
    c = mk.P["mc"]
    return mk.make_op(mk.OP_MOE_COMBINE, mk.F_FP8 if scale2 is not None else 0,
                      {c["SUMS"]: sums, c["TOPKW"]: topk_w, c["XRES"]: output, c["OUT8"]: out8,
                       c["MASK"]: mask if scale2 is not None else None, c["SCALE2"]: scale2},
                      {0: H, 1: inter, 2: ns})


def copy_layer(mk, t, input, output):
    """output = input (the debug per-layer residual snapshot; the reference's copy_layer)."""
    assert input.numel() == output.numel(), (input.shape, output.shape)
    return mk.make_op(mk.OP_COPY, 0, {0: input, 1: output}, {0: input.numel()})


def stream_layer(mk, t, weight, dummy, dummy_in=None):
    return mk.make_op(mk.OP_STREAM, 0, {0: weight, 1: dummy}, {0: weight.shape[0], 1: weight.shape[1]})


NEW_LAYERS = {
    "embed_layer": embed_layer, "linear_gemv_layer": linear_gemv_layer, "mla_prep_layer": mla_prep_layer,
    "mla_attend_layer": mla_attend_layer, "mla_merge_uv_layer": mla_merge_uv_layer,
    "moe_router_layer": moe_router_layer, "gateup_layer": gateup_layer,
    "moe_w2_combine_layer": moe_w2_combine_layer, "stream_layer": stream_layer, "copy_layer": copy_layer,
    "moe_units_layer": moe_units_layer, "moe_combine_layer": moe_combine_layer,
}


# ----------------------------------------------------------------------------
# driving the plan


def new_workspace(torch, t, device="cuda", align=0):
    """A zeroed workspace for plan tensor t (at an `align`-byte aligned address when align > 0)."""
    dt = getattr(torch, TORCH_DTYPES[t.dtype])
    if not align:
        return torch.zeros(t.shape, dtype=dt, device=device)
    return aligned_copy(torch, torch.zeros(t.shape, dtype=dt, device=device), align)


def aligned_copy(torch, t, align):
    """A copy of t whose storage starts at a multiple of `align` bytes (a power of two): the
    reference's --align-alloc re-basing of weights, capture and workspaces (harness/run_fleet.py)."""
    if not align:
        return t
    assert align & (align - 1) == 0, f"align {align} is not a power of two"
    nbytes = t.numel() * t.element_size()
    raw = torch.empty(nbytes + align, dtype=torch.uint8, device=t.device)
    off = (-raw.data_ptr()) % align
    out = raw[off:off + nbytes].view(t.dtype).view(t.shape)
    out.copy_(t)
    assert out.data_ptr() % align == 0
    return out


def allocate_workspaces(torch, plan, align=0, device="cuda"):
    """Every workspace of the plan, zeroed (the reference's --workspaces-first allocation)."""
    return {t.name: new_workspace(torch, t, device, align) for t in plan.tensors.values() if t.kind != "input"}


_REGROUPED = {}


def regrouped_w2(w2):
    """pack_weights.regroup_w2(w2), computed once per W2 tensor and dropped with it."""
    import weakref
    from fleet.pack_weights import regroup_w2
    hit = _REGROUPED.get(id(w2))
    if hit is not None and hit[0]() is w2:
        return hit[1]
    f = regroup_w2(w2)
    _REGROUPED[id(w2)] = (weakref.ref(w2), f)
    weakref.finalize(w2, _REGROUPED.pop, id(w2), None)
    return f


_FP8 = {}


def fp8_experts(w13, w2):
    """pack_weights.fp8_experts(w13, w2) as a dict (W13q, s13, W2Fq, s2), computed once per W13
    tensor and dropped with it."""
    import weakref
    from fleet.pack_weights import fp8_experts as quantize
    hit = _FP8.get(id(w13))
    if hit is not None and hit[0]() is w13:
        return hit[1]
    f = dict(zip(("W13q", "s13", "W2Fq", "s2"), quantize(w13, w2)))
    _FP8[id(w13)] = (weakref.ref(w13), f)
    weakref.finalize(w13, _FP8.pop, id(w13), None)
    return f


def make_tensors(plan, packed, capture, meta, torch, workspaces=None, device="cuda", align=0):
    """name -> torch tensor for every plan tensor: inputs attached (shape-checked), the rest zeroed."""
    host = {}
    workspaces = workspaces or {}
    for t in plan.tensors.values():
        if t.kind == "input":
            if t.source.startswith("range:"):      # constant ids start, start + 1, ...
                start = int(t.source[6:])
                src = torch.arange(start, start + t.shape[0], dtype=torch.int32, device=device)
            elif t.source.startswith("meta:"):
                src = meta[t.source[5:]]
            elif t.source.startswith("capture:"):
                src = capture[t.source[8:]]
            elif t.source.startswith("regroup_w2:"):   # the down projection regrouped by expert unit
                src = regrouped_w2(packed[t.source[11:]])
            elif t.source.startswith("fp8:"):          # fp8:<part>:<layer>, the layer's FP8 experts
                part, layer = t.source[4:].split(":")
                src = fp8_experts(packed[f"W13_{layer}"], packed[f"W2_{layer}"])[part]
            else:
                src = packed[t.source]
            assert tuple(src.shape) == t.shape, (t.name, tuple(src.shape), t.shape)
            assert src.is_contiguous(), t.name
            host[t.name] = src
        else:
            buf = workspaces.get(t.name)
            if buf is None:
                buf = new_workspace(torch, t, device, align)
            assert tuple(buf.shape) == t.shape, (t.name, tuple(buf.shape), t.shape)
            host[t.name] = buf
    return host


def call_kwargs(c, host):
    kw = {}
    for k, v in c.args.items():
        if isinstance(v, G.Rows):
            kw[k] = host[v.name][v.start:]
        elif isinstance(v, str) and v in host:
            kw[k] = host[v]
        else:
            kw[k] = v
    return kw


def make_meta(torch, s_max, prompt_ids, n_prompt, device="cuda"):
    """The meta tensors the reference's runtime reads (fleet/build_graph.py:531-547), with its
    values: step = n_prompt - 2 (the first iteration runs at n_prompt - 1), tokens[:n_prompt] the
    prompt. Only `step` and `tokens` are read by this kernel; the rest keep the reference's
    interface for its callers."""
    tokens = torch.zeros(1, s_max, dtype=torch.int64, device=device)
    tokens[0, :n_prompt] = torch.as_tensor(list(prompt_ids), dtype=torch.int64)
    return {
        "step": torch.full((1,), n_prompt - 2, dtype=torch.int32, device=device),
        "tokens": tokens,
        "input_tokens": torch.zeros(1, 1, dtype=torch.int64, device=device),
        "output_tokens": torch.zeros(1, 1, dtype=torch.int64, device=device),
        "num_new_tokens": torch.ones(1, dtype=torch.int32, device=device),
        "prompt_lengths": torch.full((1,), n_prompt, dtype=torch.int32, device=device),
        "qo_indptr_buffer": torch.tensor([0, 1], dtype=torch.int32, device=device),
        "paged_kv_indptr_buffer": torch.zeros(2, dtype=torch.int32, device=device),
        "paged_kv_indices_buffer": torch.zeros(1, dtype=torch.int32, device=device),
        "paged_kv_last_page_len_buffer": torch.zeros(1, dtype=torch.int32, device=device),
    }


def plan_json(plan):
    return {"layers": plan.layers, "head": plan.head, "debug": plan.debug, "s_max": plan.s_max,
            "debug_scores": "scores" in plan.tensors, "attend_tc": plan.attend_tc, "moe": plan.moe,
            "variants": plan.variants,
            "split": plan.split, "head_group": plan.head_group, "dims": plan.dims.to_dict(),
            "tensors": {n: {"shape": list(t.shape), "dtype": t.dtype, "kind": t.kind, "source": t.source}
                        for n, t in plan.tensors.items()},
            "calls": [{"method": c.method, "label": c.label, "status": c.status, "tasks": c.tasks,
                       "args": {k: _json_arg(v) for k, v in c.args.items()}}
                      for c in plan.calls]}


def _json_arg(v):
    """A plan argument as JSON: tuples as lists, a row range of a tensor (graph_plan.Rows) as
    {"tensor": name, "row": first row}."""
    if isinstance(v, G.Rows):
        return {"tensor": v.name, "row": v.start}
    return list(v) if isinstance(v, tuple) else v


class MPK:
    """The built graph: mk handle + tensors. compile() uploads the schedule; __call__ runs every
    iteration left until tokens is full (the reference's mpk(), one launch); launch(iters) runs a
    given number of iterations from the handle's own step counter (one launch)."""

    def __init__(self, plan, host, meta, kernel):
        self.plan = plan
        self.host = host
        self.meta = meta
        self.kernel = kernel
        self.compiled = False
        self.step = None

    def compile(self, output_dir=None, **_):
        self.kernel.finalize()
        for c, i in zip(self.plan.calls, range(len(self.plan.calls))):
            c.tasks = self.kernel.tasks(i)
        self.compiled = True
        if output_dir:
            Path(output_dir).mkdir(parents=True, exist_ok=True)
            (Path(output_dir) / "plan.json").write_text(json.dumps(plan_json(self.plan)) + "\n")

    def sync_step(self):
        """Read meta step from the device (once per __call__)."""
        self.step = int(self.meta["step"].item())

    def launch(self, iters=1, stream=None):
        assert self.compiled, "compile() first"
        if self.step is None:
            self.sync_step()
        self.kernel.launch(iters, self.step, stream, self.meta["step"])
        self.step += iters

    def decode_token(self, token_in, token_out, stream=None):
        """The next greedy token host to host: token_in (pinned int64 host tensor, the token at the
        next position) goes to the device, one launch decodes it, token_out (pinned int64 host
        tensor) receives the token after it; returns when it is there (mk_decode_token)."""
        assert self.compiled, "compile() first"
        if self.step is None:
            self.sync_step()
        self.kernel.decode_token(self.meta["tokens"][0], self.step, token_in, token_out, stream, self.meta["step"])
        self.step += 1

    def __call__(self, stream=None):
        self.sync_step()
        iters = self.plan.s_max - 2 - self.step
        assert iters >= 1, f"no iteration left (step {self.step}, s_max {self.plan.s_max})"
        self.launch(iters, stream)

    def status(self, raise_on_error=True):
        return self.kernel.status(raise_on_error)


def build(packed, capture, meta, dims=REAL_DIMS, s_max=1056, layers=27, head=True, debug=False,
          stop_after=None, debug_scores=False, tile_linears=False, attend_tasks=False, num_workers=296,
          num_schedulers=8, profiler_tensor=None, align=0, workspaces=None, fuse_norm2=False, fuse_silu=False,
          probe_before=None, fuse_norm1=False, prefetch=False, gemv_linears=False, linear_grid=None,
          head_grid=None, gemv_w13=False, merge_tasks=False, merge_halves=1, router_tasks=False,
          merge_oproj=False, argmax_slices=G.ARGMAX_SLICES, plan=None, *, split=G.SPLIT, head_group=G.HEAD_GROUP,
          num_ctas=0, device=None, trace=False, wait_timeout_s=2.0, logit_bias=False, ep=None, attend_tc=False,
          tc_parts=1, op_tasks=None, moe=None):
    """On the machine: the plan, its tensors, one library operator per call -> (mpk, host, plan).

    The positional and keyword arguments are the reference's (fleet/build_graph.py:561-567, as
    harness/run_fleet.py:543-553 passes them). The variant switches (tile_linears ... argmax_slices)
    are checked and recorded (graph_plan.mi300_variants). num_workers / num_schedulers size the
    reference's MI300X runtime (worker and scheduler blocks); this library runs one persistent CTA
    per SM (num_ctas, 0 = every SM) and schedules on the host, so they are recorded only.
    profiler_tensor is the reference runtime's event-timing buffer: per-task timing here is
    trace=True (mk_trace), so a profiler tensor is refused. probe_before inserts one of the
    reference's MI300X fault probes and is refused. align re-bases every workspace (and, in the
    reference's driver, the weights and capture through aligned_copy) on that many bytes.

    B200 keywords: split / head_group (attention partition), num_ctas, device, trace,
    wait_timeout_s (bound of every device-side wait), logit_bias (injected routing, config 3), ep
    (an fleet.ep.EpGroup: expert parallelism; every rank calls build with the same arguments and
    its own group), attend_tc (the tensor-core attention) and tc_parts (its latent-column parts per
    split). moe: "units" (one GPU's default) or "staged" (the form expert parallelism uses; see
    graph_plan.build_plan). op_tasks: {operator kind: task count} overriding the library's partition for every
    operator of that kind (the label after "L{l}.", e.g. {"router": 16}). plan: a ready plan (the
    stream probe)."""
    import torch
    from fleet import mk

    if profiler_tensor is not None:
        raise ValueError("profiler_tensor: the MI300X runtime's event timing; use trace=True (per-task "
                         "%globaltimer stamps, mk_trace) on this library")
    if probe_before:
        raise ValueError(f"probe_before={probe_before!r}: the MI300X fault probes are not part of the B200 graph")
    if plan is None:
        plan = G.build_plan(dims, s_max, layers, head, debug, debug_scores, tile_linears, attend_tasks, fuse_norm2,
                            fuse_silu, fuse_norm1, prefetch, gemv_linears, linear_grid, head_grid, gemv_w13,
                            merge_tasks, merge_halves, router_tasks, merge_oproj, argmax_slices, split=split,
                            head_group=head_group, logit_bias=logit_bias,
                            ep=None if ep is None else (ep.rank, ep.world), attend_tc=attend_tc, tc_parts=tc_parts,
                            moe=moe)
    plan.variants = dict(plan.variants, num_workers=num_workers, num_schedulers=num_schedulers, align=align)
    if ep is not None:
        workspaces = dict(workspaces or {})
        workspaces["ep_peers"] = ep.peers
    if stop_after:
        plan.truncate(stop_after)
    assert not plan.chain_violations(), f"the chain is broken: {plan.chain_violations()}"
    dev = device if device is not None else torch.cuda.current_device()
    host = make_tensors(plan, packed, capture, meta, torch, workspaces, device=f"cuda:{dev}", align=align)
    kernel = mk.MegaKernel(device=dev, num_ctas=num_ctas, trace=trace, wait_timeout_s=wait_timeout_s)
    n_cta = num_ctas or torch.cuda.get_device_properties(dev).multi_processor_count
    index = {}
    for i, c in enumerate(plan.calls):
        op = NEW_LAYERS[c.method](mk, None, **call_kwargs(c, host))
        kind = c.label.split(".", 1)[-1]
        if op_tasks and kind in op_tasks:
            op.ntasks = int(op_tasks[kind])
        if c.beside and op.ntasks == 0:
            # the operators it runs beside keep their CTAs; it takes the rest (tasks are dealt to
            # CTAs in chain order from a rotating start, so the free CTAs are the next ones). The
            # expert units take every CTA: their last tasks, on the CTAs of the operators beside,
            # run routed units only, after those operators (fleet_mk.h MK_I_MU_FTASKS)
            busy = sum(kernel.tasks(index[b]) for b in c.beside)
            if 0 < busy < n_cta:
                if c.method == "moe_units_layer":
                    op.ntasks = n_cta
                    op.ip[mk.P["mu_i"]["FTASKS"]] = n_cta - busy
                else:
                    op.ntasks = n_cta - busy
        kernel.add(op)
        index[c.label] = i
    set_plan_deps(plan, kernel)
    return MPK(plan, host, meta, kernel), host, plan


def prefill(packed, capture, meta, n_prompt, dims=REAL_DIMS, s_max=1056, layers=27, split=G.SPLIT,
            head_group=G.HEAD_GROUP, attend_tc=False, device=None, num_ctas=0, wait_timeout_s=2.0):
    """The prompt's latent cache on the GPU (the reference fills it with an HF prefill,
    harness/run_reference.py:371-377): the decode graph without the head, teacher-forced over
    positions 0 .. n_prompt - 2 in ONE launch of n_prompt - 1 iterations. Iteration i embeds the
    prompt token tokens[i] and appends cache row i of every layer, exactly as a decode step at
    that position would (the same kernels, the same arithmetic), so the cache equals the
    token-by-token reference prefill bit for bit. The decode graph then starts at position
    n_prompt - 1. Returns the launch's device status (a dict)."""
    plan = G.build_plan(dims, s_max, layers, False, split=split, head_group=head_group, attend_tc=attend_tc)
    mpk, host, plan = build(packed, capture, meta, dims, s_max, layers, False, plan=plan, device=device,
                            num_ctas=num_ctas, wait_timeout_s=wait_timeout_s)
    mpk.compile()
    mpk.kernel.launch(n_prompt - 1, -1)          # iteration i runs at position i
    st = mpk.status(raise_on_error=False)
    mpk.kernel.close()
    return st


def set_plan_deps(plan, kernel):
    """Explicit operator dependencies of the plan (labels -> operator indices)."""
    index = {c.label: i for i, c in enumerate(plan.calls)}
    for i, c in enumerate(plan.calls):
        if c.deps:
            kernel.set_deps(i, [index[d] for d in c.deps])


# ----------------------------------------------------------------------------
# dry run


class FakeTensor:
    def __init__(self, name, shape, dtype):
        self.name, self.shape, self.dtype = name, tuple(shape), dtype

    def numel(self):
        n = 1
        for s in self.shape:
            n *= s
        return n

    def dim(self):
        return len(self.shape)

    def data_ptr(self):
        return 0x10000 + (hash(self.name) & 0xFFFFFFF) * 256

    def __getitem__(self, rows):
        assert isinstance(rows, slice) and rows.step is None and rows.stop is None
        return FakeTensor(f"{self.name}[{rows.start}:]", (self.shape[0] - rows.start,) + self.shape[1:], self.dtype)


class FakeMk:
    """Records operators instead of calling the library (the reference's FakeMPK role)."""
    OP_EMBED, OP_GEMV, OP_MLA_PREP, OP_MLA_ATTEND, OP_MLA_MERGE_UV, OP_ROUTER, OP_GATEUP, OP_W2_COMBINE, OP_STREAM, \
        OP_COPY, OP_MOE_UNITS, OP_MOE_COMBINE = range(1, 13)
    F_NORM, F_RESIDUAL, F_ARGMAX, F_EXPERT, F_STATIC_IDS, F_EP, F_TC, F_FP8 = 1, 2, 4, 8, 16, 32, 64, 128

    def __init__(self):
        from fleet.mk import P
        self.P = P
        self.ops = []
        self.deps = {}

    def set_deps(self, op_index, deps):
        assert 1 <= len(deps) <= 2 and all(0 <= d < op_index for d in deps), (op_index, deps)
        self.deps[op_index] = list(deps)

    def make_op(self, type_, flags=0, ptrs=None, ips=None, fps=None, ntasks=0):
        rec = {"type": type_, "flags": flags, "ptrs": {k: (v.name if hasattr(v, "name") else v) for k, v in (ptrs or {}).items() if v is not None},
               "ips": dict(ips or {}), "fps": dict(fps or {})}
        self.ops.append(rec)
        return rec


def dry_run(dims=REAL_DIMS, s_max=1056, layers=27, head=True, debug=False, stop_after=None,
            debug_scores=False, tile_linears=False, attend_tasks=False, fuse_norm2=False, fuse_silu=False,
            probe_before=None, fuse_norm1=False, prefetch=False, gemv_linears=False, linear_grid=None,
            head_grid=None, gemv_w13=False, merge_tasks=False, merge_halves=1, router_tasks=False,
            merge_oproj=False, argmax_slices=G.ARGMAX_SLICES, plan=None, *, split=G.SPLIT,
            head_group=G.HEAD_GROUP, ep=None, attend_tc=False, moe=None):
    """The plan and every operator's parameters, without a GPU: returns (plan, recorded ops).
    Positional arguments as the reference's dry_run (fleet/build_graph.py:786-790, called
    positionally by harness/run_fleet.py:510-513); ep (rank, world): that rank's
    expert-parallel plan."""
    if probe_before:
        raise ValueError(f"probe_before={probe_before!r}: the MI300X fault probes are not part of the B200 graph")
    if plan is None:
        plan = G.build_plan(dims, s_max, layers, head, debug, debug_scores, tile_linears, attend_tasks, fuse_norm2,
                            fuse_silu, fuse_norm1, prefetch, gemv_linears, linear_grid, head_grid, gemv_w13,
                            merge_tasks, merge_halves, router_tasks, merge_oproj, argmax_slices, split=split,
                            head_group=head_group, ep=ep, attend_tc=attend_tc, moe=moe)
    if stop_after:
        plan.truncate(stop_after)
    assert not plan.chain_violations(), plan.chain_violations()
    host = {n: FakeTensor(n, t.shape, t.dtype) for n, t in plan.tensors.items()}
    fmk = FakeMk()
    for c in plan.calls:
        NEW_LAYERS[c.method](fmk, None, **call_kwargs(c, host))
    set_plan_deps(plan, fmk)
    return plan, fmk.ops


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--layers", type=int, default=27)
    ap.add_argument("--no-head", action="store_true")
    ap.add_argument("--s-max", type=int, default=1056)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    plan, ops = dry_run(REAL_DIMS, args.s_max, args.layers, not args.no_head)
    print(json.dumps(G.summary(plan)))
    if args.out:
        Path(args.out).write_text(json.dumps(plan_json(plan)) + "\n")


if __name__ == "__main__":
    main()
