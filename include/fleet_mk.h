/*
 * fleet_mk.h -- C ABI of the B200 (sm_100a) persistent decode megakernel.
 *
 * Plain C types only (pointers are device addresses the caller owns; sizes are element
 * counts); every call returns 0 on success or a negative MK_E* code, with a message from
 * mk_last_error(). One handle per device; calls on a handle are not re-entrant.
 *
 * What these entry points replace in the reference (GolfOscarr/fleet-amd-task, paths within
 * that project):
 *   - The runtime's generated C ABI: init_persistent_kernel(std::vector<void*> meta_tensors, ...),
 *     launch_persistent_kernel(cudaStream_t), finalize_persistent_kernel()
 *     (hunk headers fleet/patches/new_tasks.patch:301, :374, :384). Here the library is fixed
 *     (no per-graph code generation): mk_create / mk_add_op / mk_finalize stand for the
 *     registration plus compile() of fleet/build_graph.py:561-593 and harness/run_fleet.py:556,
 *     mk_launch for launch_persistent_kernel (mpk(), harness/run_fleet.py:590-592), mk_destroy
 *     for finalize_persistent_kernel.
 *   - The per-operator registration _new_task(mpk, grid, block, tensors, task_type, params)
 *     (fleet/build_graph.py:36-46) and the *_layer methods (fleet/build_graph.py:49-408): one
 *     mk_add_op per operator, its tensors in MkOp.ptr and its integer parameters in MkOp.ip.
 *   - The task kernels' contract (fleet/tasks/README.md "Worker contract";
 *     fleet/tasks/mi300/*.cuh *_task_impl): each MK_OP_* below names the reference task(s)
 *     whose arithmetic it carries.
 */
#ifndef FLEET_MK_H
#define FLEET_MK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define MK_ABI_VERSION 1

/* error codes */
#define MK_OK 0
#define MK_EINVAL (-1)     /* bad argument or plan */
#define MK_ECUDA (-2)      /* a CUDA runtime call failed */
#define MK_ESTATE (-3)     /* call out of order (e.g. add after finalize) */
#define MK_EDEVICE (-4)    /* the kernel reported an error in its status word */

/* device status error codes (MkStatus.error) */
#define MK_DERR_NONE 0
#define MK_DERR_WAIT_TIMEOUT 1     /* an event wait ran past MkConfig.wait_timeout_ns */
#define MK_DERR_RING_TIMEOUT 2     /* a weight-stream stage did not arrive / free in time (err_info 1:
                                      a consumer's wait, 2: the producer's, 3: a leaving producer could
                                      not drain its copies in flight; err_op and err_task are then ~0) */
#define MK_DERR_TOKEN_RANGE 3      /* a token id outside [0, V) was read (clamped) */
#define MK_DERR_ABORTED 4          /* another CTA reported an error first */
#define MK_DERR_BAD_EXPERT 5       /* a routed expert id outside [0, E_TOTAL) */

/* operator types */
enum MkOpType {
  MK_OP_EMBED = 1,        /* x_res = W_embed[tokens[pos]]                (stock embedding task) */
  MK_OP_GEMV = 2,         /* out = bf16(W (norm?(x)) (+ res)), optional fused argmax
                             (linear_gemv_mi300.cuh:143-252; lm_head + argmax_partial/reduce) */
  MK_OP_MLA_PREP = 3,     /* cache append, RoPE, ql_nope = q_nope W_uk   (mla_prep_mi300.cuh:34-139) */
  MK_OP_MLA_ATTEND = 4,   /* split-KV attention partials                 (mla_attend_mi300.cuh:48-280) */
  MK_OP_MLA_MERGE_UV = 5, /* merge of the splits, attn = o W_uv^T        (mla_merge_uv_mi300.cuh:101-344) */
  MK_OP_ROUTER = 6,       /* norm2, FP32 logits, softmax, top-k, forced  (moe_router_mi300.cuh:115-354) */
  MK_OP_GATEUP = 7,       /* mid = W13 h, act = bf16(silu(g) u) per slot (gang_moe_w13_gemv_mi300.cuh;
                             layer 0's gang_linear_silu) */
  MK_OP_W2_COMBINE = 8,   /* out8 = W2 act per slot, x += sum w out8     (gang_moe_w2_silu_mi300.cuh
                             + moe_mul_sum_add) */
  MK_OP_STREAM = 9,       /* read-only bandwidth probe of the weight ring (stream_mi300.cuh:99) */
  MK_OP_COPY = 10,        /* dst = src, n BF16 values (the debug per-layer residual snapshot, the
                             reference's copy_layer in fleet/graph_plan.py:565-567) */
  MK_OP_MOE_UNITS = 11,   /* the experts' gate/up, SwiGLU and down projection by units: a unit is
                             (slot, part p of the down projection's K, lane class q mod 8); it
                             computes the gate/up rows of its intermediates and, for every output
                             row, the down projection's level-2 butterfly subtree sum over its
                             lanes (the arithmetic of gang_moe_w13_gemv_mi300.cuh and
                             gang_moe_w2_silu_mi300.cuh, regrouped) */
  MK_OP_MOE_COMBINE = 12  /* out8 = bf16(down projection) per slot from the units' subtree sums,
                             x += sum w out8 (moe_mul_sum_add) */
};

/* MkOp.flags */
#define MK_F_NORM (1 << 0)       /* GEMV/GATEUP: RMSNorm prologue on x with ptr w_norm */
#define MK_F_RESIDUAL (1 << 1)   /* GEMV: add res before the rounding */
#define MK_F_ARGMAX (1 << 2)     /* GEMV: greedy argmax of the output into tokens[pos + 1] */
#define MK_F_EXPERT (1 << 3)     /* GATEUP: groups are the routed slots of `mask`; MOE_UNITS: the
                                    slots before FIXED0 read their experts from `mask` after the router */
#define MK_F_STATIC_IDS (1 << 4) /* GATEUP: `mask` holds constant expert ids (no wait for a router);
                                    MOE_UNITS: slot FIXED0 + k uses expert EXP0 + k (the shared
                                    experts, no wait for a router) */
#define MK_F_EP (1 << 5)         /* GATEUP / W2_COMBINE: expert parallelism by slot over N ranks, each
                                    holding every expert's weights: slot s (the TOPK routed slots,
                                    then the shared ones) is computed by rank s mod N. GATEUP spreads
                                    its rank's groups over its tasks (group g is slot SLOT0 + g).
                                    W2_COMBINE task t computes its rank's slots for its rows, stores
                                    them into every peer's exchange words, reads the other ranks'
                                    slots from its own words as they arrive (each 64-bit word carries
                                    its iteration tag) and combines all slots in slot order */
#define MK_F_TC (1 << 6)         /* MLA_ATTEND: the tensor-core form (mma.sync BF16, FP32 accumulation):
                                    one task per split for all 16 heads, cache rows streamed as TMA
                                    boxes; DC 512, DR 64, 16 heads, head group 16. Its sums run in the
                                    tensor cores' order, so its partials match the specified-order
                                    form within rounding, not bit for bit */

#define MK_F_FP8 (1 << 7)        /* MOE_UNITS / MOE_COMBINE: weight-only FP8 experts (the reference's D26):
                                    W13 and W2F hold E4M3 codes (one byte), one scale per tensor (gate,
                                    up and down of each expert); the activations are rounded to FP16
                                    (finite values beyond it saturate at +-65504) for the products,
                                    which are exact in FP32 (4 and 11 significant bits), the sums run
                                    in the BF16 form's order, and each row's total is multiplied by its
                                    tensor's scale before the BF16 rounding */

#define MK_MAX_PTRS 16
#define MK_MAX_IPARAMS 16

/* One operator. Index meaning per type (MK_P_* / MK_I_* below); unused entries 0. */
typedef struct MkOp {
  int32_t type;
  int32_t flags;
  int32_t ntasks;          /* 0: the library chooses (one task per CTA or fewer) */
  int32_t reserved;
  void* ptr[MK_MAX_PTRS];
  int64_t ip[MK_MAX_IPARAMS];
  double fp[4];
} MkOp;

/* ptr / ip indices per operator type */
enum { /* MK_OP_EMBED */ MK_P_EMB_W = 0, MK_P_EMB_TOKENS = 1, MK_P_EMB_OUT = 2,
       MK_I_EMB_V = 0, MK_I_EMB_H = 1 };
enum { /* MK_OP_GEMV */ MK_P_GEMV_X = 0, MK_P_GEMV_WNORM = 1, MK_P_GEMV_W = 2, MK_P_GEMV_RES = 3,
       MK_P_GEMV_OUT = 4, MK_P_GEMV_HOUT = 5, MK_P_GEMV_TOKENS = 6,
       MK_I_GEMV_N = 0, MK_I_GEMV_K = 1, MK_I_GEMV_VOCAB_STRIDE = 2 };
enum { /* MK_OP_MLA_PREP */ MK_P_PREP_QKVA = 0, MK_P_PREP_WKVNORM = 1, MK_P_PREP_WUKT = 2,
       MK_P_PREP_COS = 3, MK_P_PREP_SIN = 4, MK_P_PREP_CKV = 5, MK_P_PREP_KPE = 6,
       MK_P_PREP_QLNOPE = 7, MK_P_PREP_QPE = 8,
       MK_I_PREP_NH = 0, MK_I_PREP_DN = 1, MK_I_PREP_DR = 2, MK_I_PREP_DC = 3, MK_I_PREP_SMAX = 4 };
enum { /* MK_OP_MLA_ATTEND */ MK_P_ATT_QLNOPE = 0, MK_P_ATT_QPE = 1, MK_P_ATT_CKV = 2, MK_P_ATT_KPE = 3,
       MK_P_ATT_PARTIALS = 4,
       MK_P_ATT_SCORES = 5, /* optional [nh, s_max] FP32: the scaled scores of every live row (the
                               reference's debug_scores boundary B5, fleet/build_graph.py:75-81) */
       MK_I_ATT_NH = 0, MK_I_ATT_DC = 1, MK_I_ATT_DR = 2, MK_I_ATT_SMAX = 3, MK_I_ATT_SPLIT = 4,
       MK_I_ATT_HGROUP = 5, MK_I_ATT_NSPLITS = 6, MK_I_ATT_PROW = 7,
       MK_I_ATT_CPARTS = 8 /* MK_F_TC: latent-column parts per split (1, 2, 4 or 8): task (q, j) computes
                              the split's scores and softmax and the P.V columns of part q */ };
enum { /* MK_OP_MLA_MERGE_UV */ MK_P_MRG_PARTIALS = 0, MK_P_MRG_WUV = 1, MK_P_MRG_OUT = 2,
       MK_I_MRG_NH = 0, MK_I_MRG_DV = 1, MK_I_MRG_DC = 2, MK_I_MRG_SPLIT = 3, MK_I_MRG_NSPLITS = 4,
       MK_I_MRG_PROW = 5 };
enum { /* MK_OP_ROUTER */ MK_P_RT_X = 0, MK_P_RT_WNORM = 1, MK_P_RT_WGATE = 2, MK_P_RT_HOUT = 3,
       MK_P_RT_LOGITS = 4, MK_P_RT_TOPKW = 5, MK_P_RT_ROUTING = 6, MK_P_RT_MASK = 7,
       MK_P_RT_ROUTELOG = 8, MK_P_RT_BIAS = 9,
       MK_P_RT_LOGTAG = 10,  /* optional [E] 64-bit words: each logit with the iteration's tag in the high
                                half. With it, task 0 routes once every task's tagged logits are there
                                (no arrival counter) */
       MK_P_RT_MASKTAG = 11, /* optional [TOPK + NFORCED] 64-bit words: the slots' experts with the
                                iteration's tag in the high half (read by MOE_UNITS' MASKTAG) */
       MK_I_RT_H = 0, MK_I_RT_E = 1, MK_I_RT_TOPK = 2, MK_I_RT_NFORCED = 3, MK_I_RT_LAYER = 4,
       MK_I_RT_LOGSTRIDE = 5, MK_I_RT_LOGROWS = 6 };
enum { /* MK_OP_GATEUP */ MK_P_GU_X = 0, MK_P_GU_WNORM = 1, MK_P_GU_W = 2, MK_P_GU_MASK = 3,
       MK_P_GU_MID = 4, MK_P_GU_ACT = 5, MK_P_GU_HOUT = 6,
       MK_I_GU_K = 0, MK_I_GU_I = 1, MK_I_GU_GROUPS = 2, MK_I_GU_ESTRIDE = 3, MK_I_GU_NEXP = 4,
       MK_I_GU_EPRANK = 5, MK_I_GU_EPWORLD = 6, MK_I_GU_SLOT0 = 7 };
enum { /* MK_OP_W2_COMBINE */ MK_P_W2_ACT = 0, MK_P_W2_W = 1, MK_P_W2_MASK = 2, MK_P_W2_TOPKW = 3,
       MK_P_W2_XRES = 4, MK_P_W2_OUT8 = 5,
       MK_P_W2_PEERS = 6,   /* MK_F_EP: device MkEpPeers */
       MK_I_W2_H = 0, MK_I_W2_I = 1, MK_I_W2_SLOTS = 2, MK_I_W2_ESTRIDE = 3, MK_I_W2_NEXP = 4,
       MK_I_W2_TOPK = 5, MK_I_W2_EPRANK = 6, MK_I_W2_EPWORLD = 7,
       MK_I_W2_LAYER = 8 /* MK_F_EP: the exchange layer, 0 <= layer < MkEpPeers.n_layers */ };
/* MK_OP_MOE_UNITS. W13 is the packed gate/up tensor [experts][2 I][H] (row 2i gate i, 2i + 1 up i);
   W2F is the down projection [experts][H][I] regrouped by unit: per expert, per part p (of the
   KS = parts(I) parts of Lp = I / KS values), per lane class q = 0..7, the rows [H][8 nl(q)] of the
   values of lanes q, q + 8, q + 16, q + 24 that hold any (nl(q) of them: lane l holds values
   [p Lp + 8 l, + 8), l < Lp / 8), in that lane order. SUMS [NS][KS][8][H] FP32 receives, per unit and
   row r, S_q = (v_q + v_(q+16)) + (v_(q+8) + v_(q+24)) with v_l the lane's (even products + odd
   products) and +0 for a lane that holds no values: the down projection's warp butterfly up to
   its second level. A q with nl(q) = 0 is no unit (its S_q is +0).
   The operator covers slots [SLOT0, SLOT0 + NSLOTS): those from FIXED0 on have fixed experts
   (slot FIXED0 + k: expert EXP0 + k, the shared experts; MK_F_STATIC_IDS), those before FIXED0 take
   their experts from `mask` after the router (MK_F_EXPERT; the weights stream once the router is
   done). Every task takes a range of the fixed slots' units and then a range of the routed slots'
   units, each range about 1/ntasks of its kind's bytes; x (x_res) is normalised by the task itself
   (MK_F_NORM), so it needs no router output. */
enum { /* MK_OP_MOE_UNITS */ MK_P_MU_X = 0, MK_P_MU_WNORM = 1, MK_P_MU_W13 = 2, MK_P_MU_W2F = 3, MK_P_MU_MASK = 4,
       MK_P_MU_SUMS = 5, MK_P_MU_ACT = 6 /* optional [NS][I] BF16 */, MK_P_MU_HOUT = 7 /* optional */,
       MK_P_MU_MASKTAG = 8 /* optional: the router's tagged slot experts; the routed slots' weights stream
                              as soon as their words carry the iteration's tag (no wait for the router's
                              completion) */,
       MK_I_MU_H = 0, MK_I_MU_I = 1, MK_I_MU_SLOT0 = 2, MK_I_MU_NSLOTS = 3 /* slots of this operator */,
       MK_I_MU_NS = 4 /* all slots (SUMS, ACT) */, MK_I_MU_NEXP = 5, MK_I_MU_EXP0 = 6 /* MK_F_STATIC_IDS */,
       MK_I_MU_FIXED0 = 7 /* the first slot with a fixed expert (SLOT0 + NSLOTS: none) */,
       MK_I_MU_FTASKS = 8 /* the tasks [0, FTASKS) share the fixed slots' units (0, or FTASKS at least
                             the task count, which is at most the live units: every task); the
                             others run routed units only (an operator beside the router gives its
                             tasks on the router's CTAs no fixed units: they start when it is done).
                             The operator's tasks are dealt to CTAs from the rotating start, so with
                             one task per CTA the last tasks land on the CTAs of the operators just
                             before it */,
       MK_P_MU_SCALE13 = 9 /* MK_F_FP8: [experts][2] FP32, the gate and up scales */ };
/* MK_OP_MOE_COMBINE: per row r and slot s, the down projection's part sums
   ((S_0 + S_4) + (S_2 + S_6)) + ((S_1 + S_5) + (S_3 + S_7)) added in part order, rounded to BF16
   (out8), then x_res = bf16(x_res + sum_s f32(out8_s w_s)) in slot order. */
enum { /* MK_OP_MOE_COMBINE */ MK_P_MC_SUMS = 0, MK_P_MC_TOPKW = 1, MK_P_MC_XRES = 2, MK_P_MC_OUT8 = 3 /* optional */,
       MK_P_MC_MASK = 4, MK_P_MC_SCALE2 = 5 /* MK_F_FP8: the slots' experts and [experts] FP32 down scales */,
       MK_I_MC_H = 0, MK_I_MC_I = 1, MK_I_MC_NS = 2 };
/* Expert parallelism: where each rank's exchange words are, as this rank maps them (peer pointers
   opened with mk_ep_ipc_open). xch[r] is rank r's [2][n_layers][n_slots][hidden / 2] array of
   64-bit words: the low half holds two BF16 outputs (rows 2k, 2k + 1 of one slot), the high half
   the iteration tag that wrote them (the handle's exchange iteration, 1-based; halves alternate by
   its parity). A sender stores whole words (one 64-bit store each), so a reader that sees the tag
   it expects also sees the data: no fence and no separate counter. */
#define MK_EP_MAX_RANKS 8
#define MK_EP_MAX_TASKS 256
typedef struct MkEpPeers {
  uint64_t* xch[MK_EP_MAX_RANKS];
  int32_t nranks, rank;
  int32_t n_layers, n_slots, hidden;   /* the geometry the buffers were allocated for */
  int32_t reserved[3];
} MkEpPeers;
enum { /* MK_OP_STREAM */ MK_P_ST_W = 0, MK_P_ST_OUT = 1, MK_I_ST_ROWS = 0, MK_I_ST_K = 1 };
enum { /* MK_OP_COPY */ MK_P_CP_SRC = 0, MK_P_CP_DST = 1, MK_I_CP_N = 0 };

typedef struct MkConfig {
  int32_t device;            /* CUDA device ordinal */
  int32_t num_ctas;          /* 0: one per SM */
  int64_t wait_timeout_ns;   /* bound of every spin (event, stage); 0: 2 s */
  int32_t trace;             /* 1: record per-task %globaltimer stamps (mk_trace) */
  int32_t reserved[7];
} MkConfig;

typedef struct MkStatus {
  uint32_t error;            /* MK_DERR_* of the first error, 0 if none */
  uint32_t err_op;           /* operator index of the first error */
  uint32_t err_task;         /* task index within the operator */
  uint32_t err_cta;
  uint32_t err_info;         /* code-specific detail (the awaited event index, the bad id) */
  uint32_t aborted_ctas;     /* CTAs that left early after an error */
  uint64_t launches;         /* successful launches so far */
  uint64_t generation;       /* decode iterations run so far */
} MkStatus;

typedef struct MkTraceRecord {
  uint32_t op, task, cta, iter;
  uint64_t t_ready;          /* the dependency was satisfied (%globaltimer, ns) */
  uint64_t t_end;            /* the task signalled its event */
  uint64_t t_body;           /* the task's prologue (activations loaded) was done, 0 if none */
  uint64_t t_stages;         /* its last weight stage was consumed, 0 if none */
  uint64_t wait_ns;          /* time its consumer warp 0 spent waiting for weight stages */
} MkTraceRecord;

typedef struct MkHandle MkHandle;

/* Library ABI version (MK_ABI_VERSION). */
int mk_version(void);
/* Last error message of this thread (static storage). */
const char* mk_last_error(void);

/* Create a handle on cfg->device (replaces init_persistent_kernel's construction part). */
int mk_create(const MkConfig* cfg, MkHandle** out);
/* Append one operator; *op_index receives its position in the chain. Operators run in the
   order added; each waits for the previous one (the reference's chain rule,
   fleet/graph_plan.py:189-199). */
int mk_add_op(MkHandle* h, const MkOp* op, int32_t* op_index);
/* Build the per-CTA schedule and upload it (the reference's compile()). */
int mk_finalize(MkHandle* h);
/* Run `iters` decode iterations in ONE kernel launch on `stream` (a cudaStream_t, NULL for the
   default stream). Iteration i runs at position step + 1 + i: it reads tokens[step + 1 + i]
   and writes tokens[step + 2 + i]; `meta_step` (int32 device pointer or NULL) receives
   step + iters when the launch completes (the reference's prepare_next_batch, D14). MK_EINVAL if
   a position falls outside the cache rows of the plan's mla_prep operators (step + iters + 1 >=
   s_max) or step < -1: nothing is launched. */
int mk_launch(MkHandle* h, void* stream, int32_t iters, int32_t step, int32_t* meta_step);
/* One greedy token from host memory to host memory, in C (no per-token driver code between the
   copies and the launch): *token_in (pinned host int64) is copied to tokens[step + 1] on the
   device, one iteration runs at step (as mk_launch with iters 1), tokens[step + 2] is copied to
   *token_out (pinned host int64), and the call returns when the stream is done. `tokens` is the
   device int64 row the plan's embedding reads (meta tokens[0]). The host side of the reference's
   greedy loop, harness/run_reference.py:380-398, one token per call. */
int mk_decode_token(MkHandle* h, void* stream, int64_t* tokens, int32_t step, const int64_t* token_in,
                    int64_t* token_out, int32_t* meta_step);
/* Copy the device status word (synchronises the handle's last stream). MK_EDEVICE if error. */
int mk_status(MkHandle* h, MkStatus* out);
/* Clear a device error so the handle can launch again (the events are reset too). */
int mk_reset(MkHandle* h);
/* Trace records of the last launch (trace enabled): copies up to cap records, *n = count. */
int mk_trace(MkHandle* h, MkTraceRecord* out, int64_t cap, int64_t* n);
/* Expert parallelism buffers (no counterpart in the reference, which exchanged through NCCL):
   device memory that peer processes can map (cudaMalloc, zeroed), its 64-byte IPC handle, and a
   peer's buffer opened in this process (peer access enabled lazily); close and free release them.
   Every rank of a group must launch the same iteration counts: the exchange tags count the
   handle's iterations since mk_finalize (a failed launch consumes its iterations too, and
   mk_reset keeps the count), so the ranks' tags stay equal. */
int mk_ep_alloc(int32_t device, size_t bytes, void** dev_ptr);
int mk_ep_free(void* dev_ptr);
int mk_ep_ipc_handle(void* dev_ptr, void* handle64);
int mk_ep_ipc_open(int32_t device, const void* handle64, void** peer_ptr);
int mk_ep_ipc_close(void* peer_ptr);

/* Replace the consumer-side dependencies of operator op_index (by default: the previous
   operator) with n (1 or 2) earlier operators of the same iteration; before mk_finalize. Every
   operator must still lead to the last one. Lets independent operators overlap (the MoE's
   shared experts run beside the router). */
int mk_set_op_deps(MkHandle* h, int32_t op_index, const int32_t* dep_ops, int32_t n);
/* Schedule introspection: tasks of operator op_index, and the CTA of its task t. */
int mk_op_tasks(MkHandle* h, int32_t op_index, int32_t* ntasks);
/* Release everything the library allocated (replaces finalize_persistent_kernel). */
int mk_destroy(MkHandle* h);

/* Test hook: make operator op_index of the next launch wait for an event that never fires,
   so the bounded wait runs out and the status reports MK_DERR_WAIT_TIMEOUT (no GPU fault). */
int mk_debug_block_op(MkHandle* h, int32_t op_index);

/* Self-test of the device's deterministic arithmetic on n values (device pointers):
   fn 0 det_exp, 1 det_log, 2 silu, 3 bf16_from_f64 (x is double*, out is uint16_t*),
   4 bf16 round of float (out uint16_t*). */
int mk_selftest_math(int32_t fn, const void* x, void* out, int64_t n, void* stream);

/* MLA decode attention without any device allocation. There is no counterpart in the reference;
   it exists for callers that cannot call cudaMalloc where they call this (an engine that owns all
   of HBM through its own pool, code running under the caller's allocator lock, loops that cannot
   take cudaMalloc's implicit synchronisation). It computes what the persistent kernel's
   MK_OP_MLA_ATTEND + MK_OP_MLA_MERGE_UV compute at position `pos`, bit for bit:
   attn_out[nh * d_v] = merge of the ceil((pos + 1) / split) live splits, times W_uv.
   Inputs (device, BF16): ql_nope [nh, d_c], q_pe [nh, d_r], c_kv [>= pos + 1, d_c],
   k_pe [>= pos + 1, d_r], w_uv [nh, d_v, d_c]. The split-KV partials live in a file-scope
   __device__ array of 2 MiB (64 splits x 16 heads x 516 floats) that each GPU keeps until the
   process exits: limits nh <= 16, d_c <= 512 (a multiple of 32), d_r <= 64 (even), split <= 256,
   and ceil((pos + 1) / split) <= 64; anything beyond returns MK_EINVAL. The first call on a
   device looks up that array's device address (cudaGetSymbolAddress) and should come before any
   stream capture. All calls share the array: calls that overlap on the GPU race. */
int mk_mla_decode_noalloc(const void* ql_nope, const void* q_pe, const void* c_kv, const void* k_pe,
                          const void* w_uv, void* attn_out, int32_t nh, int32_t d_c, int32_t d_r, int32_t d_v,
                          int32_t pos, int32_t split, float softmax_scale, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* FLEET_MK_H */
