"""The decode task graph as data: the operator chain of one greedy decode token, the tensors it
attaches or allocates, and the parameters of every operator.

Same entry points and data model as the reference's fleet/graph_plan.py (Tensor, Call, Plan,
OUTPUT_ARGS, build_plan, the chain rule :189-199, truncate, summary, partials_row), with the
B200 operator set of include/fleet_mk.h. Per token the chain is

    prologue.embed
    per layer l:  L{l}.qkva        GEMV, input RMSNorm fused (reference: norm1 + qkva)
                  L{l}.mla_prep    cache append at the step row, RoPE, ql_nope = q_nope W_uk
                  L{l}.mla_attend  split-KV partials over (head group, split) tasks
                  L{l}.mla_merge_uv  merge of the live splits, attn = o W_uv^T
                  L{l}.o_proj      GEMV + residual into x_res
      layer 0:    L0.gate_up       post-attention RMSNorm + gate/up GEMV + SwiGLU (dense, I 10,944)
                  L0.down          GEMV + residual (K 10,944, split over the eight warps)
      MoE layers: L{l}.router      post-attention RMSNorm + FP32 router + top-k + forced shared experts
                  L{l}.experts     (moe="units", one GPU) the expert units: per task its own RMSNorm of
                                   x_res, its share of the shared slots' units (no wait for the
                                   router), then its share of the routed slots' units; a unit runs
                                   gate/up + SwiGLU of its intermediates and its lanes' part of the
                                   down projection (butterfly subtree sums)
                  L{l}.combine     the down projection per slot from the subtree sums + the weighted
                                   combine into x_res
                  or (moe="staged", and with expert parallelism):
                  L{l}.w13s        the shared experts' gate/up + SwiGLU (own RMSNorm; waits for o_proj
                                   only, so it runs beside the router)
                  L{l}.w13r        gate/up GEMV + SwiGLU of the TOPK routed slots (waits for the router)
                  L{l}.w2_combine  down GEMV of the 8 slots + the weighted combine into x_res
    head.lm_head  GEMV with the final RMSNorm, and the greedy argmax into tokens[pos + 1]

against the reference's final stack (fleet/graph_plan.py:416-602 with harness/run_fleet.py:291-298)
the norm1/norm2/silu/combine/argmax operators are fused into their neighbours: 217 operators per
token at 27 layers with the expert units, 243 staged (the reference: 246). Operators wait for the
previous one unless a call lists its `deps` (the shared-expert branch).
"""
import struct
from dataclasses import dataclass, field

from fleet.pack_weights import Dims, REAL_DIMS, unit_parts

SPLIT = 128            # latent-cache rows per attention split task
HEAD_GROUP = None      # query heads per attention task; None: auto_head_group (1 at 1K context)
PLAN_CTAS = 148        # the CTAs (SMs of one B200) the automatic head group fills
ROUTE_LOG_ROWS = 32    # the reference's route_log [32, L - 1, 8] (fleet/graph_plan.py:376)
RMS_EPS = 1e-6
SOFTMAX_SCALE = 0.1147213867929261
ROUTED_SCALING = 1.0


def float_bits(x: float) -> int:
    """A float parameter as its IEEE-754 bit pattern (the reference passes floats this way)."""
    return struct.unpack("<i", struct.pack("<f", x))[0]


EP_PEERS_WORDS = 24          # sizeof(MkEpPeers) / 4


def ep_slots(rank, world, n_slots):
    """The slots rank `rank` of `world` computes under expert parallelism by slot: s mod world =
    rank over all n_slots slots (the TOPK routed ones, then the shared ones). Every rank holds every
    expert's weights, so a token's eight slots spread over the ranks whatever experts the router
    picks: each rank gets ceil or floor of 8 / world."""
    assert 1 <= world and 0 <= rank < world, (rank, world)
    return [s for s in range(n_slots) if s % world == rank]


def partials_row(d_c):
    """Innermost width of the split-KV partials: D_C values of o, the lse at column D_C, padded to a
    multiple of 4 floats so every [split, head] row is 16-byte aligned (513 -> 516 at D_C 512)."""
    return ((d_c + 1 + 3) // 4) * 4


@dataclass
class Tensor:
    name: str
    shape: tuple
    dtype: str = "bf16"           # bf16 | f32 | i32 | i64
    kind: str = "new"             # new (allocated, zeroed) | input (attached: weights, capture, meta)
    source: str = ""              # inputs: "packed key", "capture:<name>" or "meta:<name>"

    @property
    def num_dims(self):
        return len(self.shape)

    def dim(self, i):
        return self.shape[i]


@dataclass
class Call:
    method: str
    args: dict
    tasks: int = 0                # filled by build_graph from the library's partition
    status: str = "new"
    note: str = ""
    label: str = ""
    deps: tuple = ()              # labels of the operators it waits for (empty: the previous one)
    beside: tuple = ()            # labels of operators it runs beside: it takes the CTAs they leave free


@dataclass(frozen=True)
class Rows:
    """Argument value: the rows [start:] of plan tensor `name` (an operator writing part of it)."""
    name: str
    start: int


# Which argument names of each method are outputs (the rest are inputs). Every operator must read
# a tensor its predecessor wrote (the reference runtime's chain rule, register_mugraph).
OUTPUT_ARGS = {
    "embed_layer": ["output"],
    "linear_gemv_layer": ["output", "h_out", "tokens_out"],
    "mla_prep_layer": ["c_kv", "k_pe", "ql_nope", "q_pe"],
    "mla_attend_layer": ["partials", "scores"],
    "mla_merge_uv_layer": ["output"],
    "moe_router_layer": ["h", "topk_w", "routing", "mask", "logits", "route_log", "logit_tag", "mask_tag"],
    "gateup_layer": ["act", "mid", "h_out"],
    "moe_w2_combine_layer": ["output", "out8"],
    "moe_units_layer": ["sums", "act", "h_out"],
    "moe_combine_layer": ["output", "out8"],
    "stream_layer": ["dummy"],
    "copy_layer": ["output"],
}


def _tensor_args(call, names):
    out = set()
    for k in names:
        v = call.args.get(k)
        if v is None:
            continue
        for x in (v if isinstance(v, (tuple, list)) else [v]):
            out.add(x.name if isinstance(x, Rows) else x)
    return out


@dataclass
class Plan:
    dims: Dims
    s_max: int
    layers: int
    head: bool
    debug: bool = False
    split: int = SPLIT
    head_group: int = HEAD_GROUP
    attend_tc: bool = False
    moe: str = "staged"
    variants: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    calls: list = field(default_factory=list)

    def t(self, name, shape, dtype="bf16", kind="new", source=""):
        assert name not in self.tensors, name
        self.tensors[name] = Tensor(name, tuple(shape), dtype, kind, source)
        return name

    def op(self, method, label, note="", deps=(), beside=(), **args):
        self.calls.append(Call(method, args, 0, "new", note, label, tuple(deps), tuple(beside)))

    def index_of(self, label):
        for i, c in enumerate(self.calls):
            if c.label == label:
                return i
        raise KeyError(label)

    def truncate(self, stop_label):
        """Keep the calls up to and including the labelled operator (the reference's --stop-after)."""
        self.calls = self.calls[: self.index_of(stop_label) + 1]
        return self

    def dep_labels(self, i):
        """The operators call i waits for: its explicit deps, else the previous call."""
        c = self.calls[i]
        if c.deps:
            return list(c.deps)
        return [self.calls[i - 1].label] if i > 0 else []

    def chain_violations(self):
        """Every operator must read a tensor that each operator it waits for wrote."""
        bad = []
        by_label = {c.label: c for c in self.calls}
        for i, cur in enumerate(self.calls):
            ins = _tensor_args(cur, [k for k in cur.args if k not in OUTPUT_ARGS[cur.method]])
            for d in self.dep_labels(i):
                prev = by_label[d]
                if not (_tensor_args(prev, OUTPUT_ARGS[prev.method]) & ins):
                    bad.append((prev.label, cur.label))
        return bad

    @property
    def n_ops(self):
        return len(self.calls)

    @property
    def n_tasks(self):
        return sum(c.tasks for c in self.calls)

    @property
    def n_splits(self):
        return -(-self.s_max // self.split)


def auto_head_group(n_heads: int, n_splits: int, ctas: int = PLAN_CTAS, d_c: int = 512, d_r: int = 64) -> int:
    """The largest power-of-two head group that still leaves at least one attention task per CTA.
    A task streams its split's cache rows once and runs its heads over them two at a time, so at
    long context (8K: 65 splits x 16 heads) a group of 4 saves three quarters of the per-task
    overhead and of the cache streaming; at 1K context (9 splits) every head keeps its own task.
    Groups above 1 exist for the model's latent widths (d_c 512, d_r 64) only."""
    if (d_c, d_r) != (512, 64):
        return 1
    g = 1
    while n_heads % (2 * g) == 0 and (n_heads // (2 * g)) * n_splits >= ctas:
        g *= 2
    return g


ARGMAX_SLICES = 50     # the reference's argmax_partial slice count (its D13); here the argmax is fused


def mi300_variants(tile_linears=False, attend_tasks=False, fuse_norm2=False, fuse_silu=False, fuse_norm1=False,
                   prefetch=False, gemv_linears=False, linear_grid=None, head_grid=None, gemv_w13=False,
                   merge_tasks=False, merge_halves=1, router_tasks=False, merge_oproj=False,
                   argmax_slices=ARGMAX_SLICES):
    """The reference's graph-variant switches (fleet/graph_plan.py:261-267, harness/run_fleet.py
    --tile-linears ... --merge-oproj), checked and recorded. Each selects one of its MI300X kernel
    forms or task grids; the B200 graph has one form of each operator, with what the switches turn
    on always done (the norms, the SwiGLU and the argmax fused into their GEMVs, every linear a
    GEMV, the experts' gate/up a GEMV, the router a last-arriver task, the merge in head tasks) and
    the grids chosen by the library. So the values change no operator; they are kept in the plan
    (plan.variants, plan_json) for the run records."""
    for name, v in (("linear_grid", linear_grid), ("head_grid", head_grid)):
        if v is not None and (not isinstance(v, int) or v < 1):
            raise ValueError(f"{name}: a positive task count or None, not {v!r}")
    if merge_halves not in (1, 2):
        raise ValueError(f"merge_halves: 1 or 2, not {merge_halves!r}")
    if merge_halves != 1 and not merge_tasks:
        raise ValueError("merge_halves > 1 needs merge_tasks (the reference's rule)")
    if not isinstance(argmax_slices, int) or argmax_slices < 1:
        raise ValueError(f"argmax_slices: a positive count, not {argmax_slices!r}")
    return dict(tile_linears=bool(tile_linears), attend_tasks=bool(attend_tasks), fuse_norm2=bool(fuse_norm2),
                fuse_silu=bool(fuse_silu), fuse_norm1=bool(fuse_norm1), prefetch=bool(prefetch),
                gemv_linears=bool(gemv_linears), linear_grid=linear_grid, head_grid=head_grid,
                gemv_w13=bool(gemv_w13), merge_tasks=bool(merge_tasks), merge_halves=merge_halves,
                router_tasks=bool(router_tasks), merge_oproj=bool(merge_oproj), argmax_slices=argmax_slices)


def build_plan(dims: Dims = REAL_DIMS, s_max: int = 1056, layers: int = 27, head: bool = True,
               debug: bool = False, debug_scores: bool = False, tile_linears: bool = False,
               attend_tasks: bool = False, fuse_norm2: bool = False, fuse_silu: bool = False,
               fuse_norm1: bool = False, prefetch: bool = False, gemv_linears: bool = False,
               linear_grid: int = None, head_grid: int = None, gemv_w13: bool = False, merge_tasks: bool = False,
               merge_halves: int = 1, router_tasks: bool = False, merge_oproj: bool = False,
               argmax_slices: int = ARGMAX_SLICES, *, split: int = SPLIT, head_group: int = HEAD_GROUP,
               route_log_rows: int = ROUTE_LOG_ROWS, logit_bias: bool = False, softmax_scale: float = None,
               ep: tuple = None, attend_tc: bool = False, tc_parts: int = 1, moe: str = None) -> Plan:
    """The operator chain for `layers` layers (+ the head), with the reference's positional
    arguments (fleet/graph_plan.py:261-267; the variant switches from tile_linears on are
    checked and recorded, see mi300_variants). debug: a per-layer residual snapshot
    dbg_x_res_{l} after every layer, read by the next layer (the reference's debug graph).
    debug_scores: the attention also writes its scaled scores [NH, s_max] (boundary B5).
    logit_bias: every router adds an injected FP32 bias [E] to its logits (the skewed/uniform
    routing of config 3). softmax_scale: default q_head_dim^-0.5 times the YaRN mscale^2 of the
    dims (0.1147213867929261 at REAL_DIMS).
    ep (rank, world): expert parallelism by slot (fleet/ep.py): this rank's gate/up operators and
    down projection cover the slots s (routed, then shared) with s mod world = rank; each
    down-projection task exchanges its rows with the same task of every peer before it combines.
    attend_tc: the MLA attention on the tensor cores (one task per split for all heads, FP32
    accumulation in the tensor cores' order: within rounding of the specified-order form);
    tc_parts: its latent-column parts per split (one task each).
    moe: "units" (the default on one GPU): the experts as units (slot, down-projection part, lane
    class) that each run gate/up, SwiGLU and their share of the down projection, every task the
    shared slots' units first and the routed slots' once the router is done, then a combine;
    "units_fp8": the same with weight-only FP8 experts (E4M3 codes, one scale per gate, up and
    down tensor of each expert, fleet_mk.h MK_F_FP8); "staged" (the default, and the only form,
    with ep): gate/up of the shared and of the routed slots, then the down projection and combine
    over all slots."""
    if moe is None:
        moe = "units" if ep is None else "staged"
    if moe not in ("units", "units_fp8", "staged") or (moe != "staged" and ep is not None):
        raise ValueError(f"moe={moe!r}: 'units' or 'units_fp8' (one GPU), or 'staged'")
    units = moe in ("units", "units_fp8")
    variants = mi300_variants(tile_linears, attend_tasks, fuse_norm2, fuse_silu, fuse_norm1, prefetch, gemv_linears,
                              linear_grid, head_grid, gemv_w13, merge_tasks, merge_halves, router_tasks,
                              merge_oproj, argmax_slices)
    from fleet.capture import softmax_scale as yarn_softmax_scale
    d = dims
    scale = yarn_softmax_scale(d.D_N, d.D_R) if softmax_scale is None else softmax_scale
    assert 1 <= layers <= d.L
    if attend_tc:
        head_group = d.NH
    elif head_group is None:
        head_group = auto_head_group(d.NH, -(-s_max // split), d_c=d.D_C, d_r=d.D_R)
    assert d.NH % head_group == 0
    p = Plan(d, s_max, layers, head, debug, split, head_group, attend_tc, moe)
    p.variants = variants
    n_splits = p.n_splits
    # ---- meta, capture and shared activations
    p.t("tokens", (1, s_max), "i64", "input", "meta:tokens")
    p.t("W_embed", (d.V, d.H), kind="input", source="W_embed")
    p.t("cos", (s_max, d.D_R), kind="input", source="capture:cos")
    p.t("sin", (s_max, d.D_R), kind="input", source="capture:sin")
    p.t("x_res", (1, d.H))
    p.t("h", (1, d.H))
    p.t("qkva", (1, d.QKVA_OUT))
    p.t("ql_nope", (d.NH, d.D_C))
    p.t("q_pe", (d.NH, d.D_R))
    p.t("partials", (n_splits, d.NH, partials_row(d.D_C)), "f32")
    if debug_scores:
        p.t("scores", (d.NH, s_max), "f32")
    if debug:
        for l in range(layers):
            p.t(f"dbg_x_res_{l}", (1, d.H))
    p.t("attn", (1, d.NH * d.D_V))
    if layers >= 1:
        p.t("mid0", (1, 2 * d.I_DENSE))
        p.t("act0", (1, d.I_DENSE))
    if layers >= 2:
        p.t("topk_w", (1, d.N_SLOTS), "f32")
        p.t("routing", (d.E_TOTAL,), "i32")
        p.t("mask", (d.E_TOTAL + 1,), "i32")
        p.t("mask_shared", (d.N_SHARED,), "i32", "input", f"range:{d.E}")
        p.t("logits_router", (1, d.E), "f32")
        p.t("mid", (d.N_SLOTS, 2 * d.I_MOE))
        p.t("act8", (d.N_SLOTS, d.I_MOE))
        p.t("out8", (d.N_SLOTS, d.H))
        if units:
            p.t("moe_sums", (d.N_SLOTS, unit_parts(d.I_MOE), 8, d.H), "f32")
            p.t("logit_tag", (d.L - 1, d.E), "i64")          # per MoE layer: tagged-word hand-offs
            p.t("mask_tag", (d.L - 1, d.N_SLOTS), "i64")
        p.t("route_log", (route_log_rows, d.L - 1, d.N_SLOTS), "i32")
        if ep is not None:
            p.t("ep_peers", (EP_PEERS_WORDS,), "i32")
    p.op("embed_layer", "prologue.embed", input="tokens", weight="W_embed", output="x_res")
    for l in range(layers):
        p.t(f"w_norm1_{l}", (d.H,), kind="input", source=f"w_norm1_{l}")
        p.t(f"w_norm2_{l}", (d.H,), kind="input", source=f"w_norm2_{l}")
        p.t(f"W_qkva_{l}", (d.QKVA_OUT, d.H), kind="input", source=f"W_qkva_{l}")
        p.t(f"w_kv_norm_{l}", (d.D_C,), kind="input", source=f"w_kv_norm_{l}")
        p.t(f"W_ukT_{l}", (d.NH, d.D_C, d.D_N), kind="input", source=f"W_ukT_{l}")
        p.t(f"W_uv_{l}", (d.NH, d.D_V, d.D_C), kind="input", source=f"W_uv_{l}")
        p.t(f"W_o_{l}", (d.H, d.NH * d.D_V), kind="input", source=f"W_o_{l}")
        p.t(f"c_kv_{l}", (s_max, d.D_C), kind="input", source=f"capture:c_kv_{l}")
        p.t(f"k_pe_{l}", (s_max, d.D_R), kind="input", source=f"capture:k_pe_{l}")
        # under debug, the layer reads the previous layer's snapshot (the same values), so the chain
        # runs through it (the reference's debug graph, fleet/graph_plan.py:433-435)
        x_in = f"dbg_x_res_{l - 1}" if debug and l > 0 else "x_res"
        p.op("linear_gemv_layer", f"L{l}.qkva", input=x_in, w_norm=f"w_norm1_{l}", weight=f"W_qkva_{l}",
             output="qkva", h_out="h", norm=True, eps=RMS_EPS)
        p.op("mla_prep_layer", f"L{l}.mla_prep", qkva="qkva", w_kv_norm=f"w_kv_norm_{l}", w_ukT=f"W_ukT_{l}",
             cos="cos", sin="sin", c_kv=f"c_kv_{l}", k_pe=f"k_pe_{l}", ql_nope="ql_nope", q_pe="q_pe", eps=RMS_EPS)
        p.op("mla_attend_layer", f"L{l}.mla_attend", ql_nope="ql_nope", q_pe="q_pe", c_kv=f"c_kv_{l}",
             k_pe=f"k_pe_{l}", partials="partials", softmax_scale=scale, split=split, n_splits=n_splits,
             head_group=head_group, tc=attend_tc, col_parts=tc_parts if attend_tc else 1,
             **(dict(scores="scores") if debug_scores else {}))
        p.op("mla_merge_uv_layer", f"L{l}.mla_merge_uv", partials="partials", w_uv=f"W_uv_{l}", output="attn",
             split=split, n_splits=n_splits)
        p.op("linear_gemv_layer", f"L{l}.o_proj", input="attn", weight=f"W_o_{l}", residual="x_res",
             output="x_res", residual_add=True)
        if l == 0:
            p.t("W_gu_0", (2 * d.I_DENSE, d.H), kind="input", source="W_gu_0")
            p.t("W_down_0", (d.H, d.I_DENSE), kind="input", source="W_down_0")
            p.op("gateup_layer", "L0.gate_up", input="x_res", w_norm="w_norm2_0", weight="W_gu_0", mid="mid0",
                 act="act0", h_out="h", groups=1, expert=False, norm=True, eps=RMS_EPS, inter=d.I_DENSE)
            p.op("linear_gemv_layer", "L0.down", input="act0", weight="W_down_0", residual="x_res", output="x_res",
                 residual_add=True)
        else:
            p.t(f"W_gate_{l}", (d.E, d.H), kind="input", source=f"W_gate_{l}")
            if moe != "units_fp8":
                p.t(f"W13_{l}", (d.E_TOTAL, 2 * d.I_MOE, d.H), kind="input", source=f"W13_{l}")
            if moe == "units_fp8":   # the experts' E4M3 codes and scales, quantised from W13 / W2
                p.t(f"W13Q_{l}", (d.E_TOTAL, 2 * d.I_MOE, d.H), "u8", "input", f"fp8:W13q:{l}")
                p.t(f"S13_{l}", (d.E_TOTAL, 2), "f32", "input", f"fp8:s13:{l}")
                p.t(f"W2FQ_{l}", (d.E_TOTAL, d.H * d.I_MOE), "u8", "input", f"fp8:W2Fq:{l}")
                p.t(f"S2_{l}", (d.E_TOTAL,), "f32", "input", f"fp8:s2:{l}")
            elif moe == "units":
                p.t(f"W2F_{l}", (d.E_TOTAL, d.H * d.I_MOE), kind="input", source=f"regroup_w2:W2_{l}")
            else:
                p.t(f"W2_{l}", (d.E_TOTAL, d.H, d.I_MOE), kind="input", source=f"W2_{l}")
            bias = {}
            if logit_bias:
                p.t(f"router_bias_{l}", (d.E,), "f32", kind="input", source=f"capture:router_bias_{l}")
                bias = dict(bias=f"router_bias_{l}")
            tags = dict(logit_tag=Rows("logit_tag", l - 1), mask_tag=Rows("mask_tag", l - 1)) if units else {}
            p.op("moe_router_layer", f"L{l}.router", input="x_res", w_norm=f"w_norm2_{l}", w_gate=f"W_gate_{l}",
                 h="h", topk_w="topk_w", routing="routing", mask="mask", logits="logits_router",
                 route_log="route_log", layer_index=l - 1, topk=d.TOPK, n_experts=d.E, n_forced=d.N_SHARED,
                 scaling=ROUTED_SCALING, eps=RMS_EPS, **bias, **tags)
            if units:
                # the expert units (fleet_mk.h MK_OP_MOE_UNITS), on the CTAs the router leaves free:
                # every task normalises x_res itself, runs its share of the shared slots' units at
                # once and its share of the routed slots' units when the router's expert ids are out;
                # the combine adds all slots
                p.op("moe_units_layer", f"L{l}.experts", deps=(f"L{l}.o_proj",), beside=(f"L{l}.router",),
                     input="x_res",
                     w_norm=f"w_norm2_{l}", mask="mask", sums="moe_sums",
                     act="act8", slot0=0, nslots=d.N_SLOTS, fixed0=d.TOPK, static_experts=d.E, norm=True,
                     mask_tag=Rows("mask_tag", l - 1), inter=d.I_MOE, eps=RMS_EPS,
                     **(dict(w13=f"W13Q_{l}", w2f=f"W2FQ_{l}", scale13=f"S13_{l}") if moe == "units_fp8"
                        else dict(w13=f"W13_{l}", w2f=f"W2F_{l}")))
                p.op("moe_combine_layer", f"L{l}.combine", deps=(f"L{l}.experts", f"L{l}.router"),
                     sums="moe_sums", topk_w="topk_w", residual="x_res", output="x_res", out8="out8", inter=d.I_MOE,
                     **(dict(mask="mask", scale2=f"S2_{l}") if moe == "units_fp8" else {}))
                if debug:
                    p.op("copy_layer", f"L{l}.snapshot", note="debug only: per-layer residual snapshot",
                         input="x_res", output=f"dbg_x_res_{l}")
                continue
            # the shared experts (slots TOPK..) need no routing: they run beside the router, on
            # their own RMSNorm of x_res
            ep_s = {} if ep is None else dict(ep=(ep[0], ep[1], d.TOPK))
            p.op("gateup_layer", f"L{l}.w13s", deps=(f"L{l}.o_proj",), beside=(f"L{l}.router",), input="x_res",
                 w_norm=f"w_norm2_{l}",
                 weight=f"W13_{l}", mask="mask_shared", mid=Rows("mid", d.TOPK), act=Rows("act8", d.TOPK),
                 groups=d.N_SHARED, expert=True, static_ids=True, norm=True, eps=RMS_EPS, inter=d.I_MOE, **ep_s)
            if ep is None:
                p.op("gateup_layer", f"L{l}.w13r", deps=(f"L{l}.router",), input="h", weight=f"W13_{l}",
                     mask="mask", mid="mid", act="act8", groups=d.TOPK, expert=True, norm=False, inter=d.I_MOE)
                p.op("moe_w2_combine_layer", f"L{l}.w2_combine", deps=(f"L{l}.w13r", f"L{l}.w13s"), input="act8",
                     weight=f"W2_{l}", mask="mask", topk_w="topk_w", residual="x_res", output="x_res", out8="out8")
            else:
                p.op("gateup_layer", f"L{l}.w13r", deps=(f"L{l}.router",), input="h", weight=f"W13_{l}",
                     mask="mask", mid="mid", act="act8", groups=d.TOPK, expert=True, norm=False, inter=d.I_MOE,
                     ep=(ep[0], ep[1], 0))
                p.op("moe_w2_combine_layer", f"L{l}.w2_combine", deps=(f"L{l}.w13r", f"L{l}.w13s"), input="act8",
                     weight=f"W2_{l}", mask="mask", topk_w="topk_w", residual="x_res", output="x_res",
                     ep=tuple(ep), peers="ep_peers", topk=d.TOPK, layer=l - 1)
        if debug:
            p.op("copy_layer", f"L{l}.snapshot", note="debug only: per-layer residual snapshot", input="x_res",
                 output=f"dbg_x_res_{l}")
    if head:
        p.t("w_final_norm", (d.H,), kind="input", source="w_final_norm")
        p.t("W_lm", (d.V, d.H), kind="input", source="W_lm")
        p.t("logits", (1, d.V))
        p.op("linear_gemv_layer", "head.lm_head", input=f"dbg_x_res_{layers - 1}" if debug else "x_res",
             w_norm="w_final_norm", weight="W_lm",
             output="logits", h_out="h", tokens_out="tokens", norm=True, argmax=True, eps=RMS_EPS)
    return p


def build_stream_plan(ops: int, rows: int, k: int = 2048, dims: Dims = REAL_DIMS) -> Plan:
    """The bandwidth probe (the reference's stream graph, fleet/graph_plan.py:647-681): `ops`
    operators, each streaming its own [rows, k] BF16 tensor through the weight ring with no
    arithmetic, so the ring's read rate is measured with the runtime's scheduling around it."""
    p = Plan(dims, 1, 0, False)
    p.t("stream_dummy", (1, 4), "i32")
    for i in range(ops):
        p.t(f"stream_w_{i}", (rows, k))
        p.op("stream_layer", f"S{i}.stream", weight=f"stream_w_{i}", dummy="stream_dummy", dummy_in="stream_dummy")
    return p


def summary(p: Plan) -> dict:
    ib = 0
    for t in p.tensors.values():
        if t.kind == "input":
            n = 1
            for s in t.shape:
                n *= s
            ib += n * {"bf16": 2, "f32": 4, "i32": 4, "i64": 8, "u8": 1}[t.dtype]
    return {"ops": p.n_ops, "tasks": p.n_tasks, "tensors_new": sum(t.kind == "new" for t in p.tensors.values()),
            "tensors_input": sum(t.kind == "input" for t in p.tensors.values()), "input_bytes": ib,
            "n_splits": p.n_splits}
