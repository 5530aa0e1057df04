// mk_runtime.cu -- host side of the persistent decode kernel and the C ABI of include/fleet_mk.h.
//
// The host owns the schedule: mk_add_op partitions each operator into tasks (row ranges of its
// weight, head-group x split pairs of the attention) and mk_finalize deals the tasks to the CTAs
// in chain order, uploads the tables and allocates the library's own device state (event
// counters, arrival counters, argmax partials, status word, trace buffer). Caller tensors are
// only ever referenced by pointer.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/fleet_mk.h"
#include "mk_kernel.cuh"

using namespace mk;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define MK_CUDA(call)                                                                       \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return fail(MK_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

}  // namespace

namespace mk {
// the error message of mk_last_error() for the library's other translation units
int set_last_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace mk

struct MkHandle {
  MkConfig cfg{};
  int num_ctas = 0;
  int num_sms = 0;
  bool finalized = false;
  int variant = KV_SHORT;   // the kernel variant the plan's operators need (KV_*)
  std::vector<OpDev> ops;
  std::vector<TaskDev> tasks;
  std::vector<std::vector<uint32_t>> cta_tasks;
  std::vector<std::vector<int32_t>> deps;   // per operator: explicit consumer dependencies (empty: previous)
  // device state
  OpDev* d_ops = nullptr;
  uint32_t* d_cta_off = nullptr;
  CtaTask* d_ctask = nullptr;
  uint32_t* d_events = nullptr;
  uint32_t* d_arrive = nullptr;
  DevStatus* d_status = nullptr;
  float* d_amax_val = nullptr;
  int32_t* d_amax_idx = nullptr;
  MkTraceRecord* d_trace = nullptr;
  uint32_t* d_trace_count = nullptr;
  uint32_t trace_cap = 0;
  uint64_t gen = 1;          // generation of the next iteration
  uint32_t ep_gen = 1;       // expert-parallel exchange tag of the next iteration (never restarts)
  uint64_t launches = 0;
  int block_op = -1;
  cudaStream_t last_stream = nullptr;
  int rr = 0;                // rotating CTA offset for operators with few tasks
  int n_tc = 0;              // tensor-core attention operators (two tensor maps each)
  int64_t cache_rows = 0;    // the fewest cache rows of the plan's cache appends (0: none): a
                             // launch's positions must stay below it
  void* d_tmaps = nullptr;
  std::vector<uint16_t> units;   // the expert-unit operators' per-task unit lists
  uint16_t* d_units = nullptr;
  // words tagged with the iteration generation (the router's tagged logits and slot experts):
  // cleared whenever the generation restarts, so no stale word carries a current tag
  std::vector<std::pair<void*, size_t>> tagged;
};

// ---------------------------------------------------------------------------------------------
// partitioning

namespace {

inline int div_up(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// rows per ring stage for rows of `row_bytes`: the most that fit
int rows_per_stage(int64_t row_bytes) {
  return std::max((int)(STAGE_BYTES / row_bytes), 1);
}

// split `n` units into `t` contiguous ranges as even as possible, each a multiple of `q` units
// except the last
void split_even(std::vector<std::pair<int, int>>& out, int n, int t, int q = 1) {
  out.clear();
  const int blocks = div_up(n, q);
  t = std::max(1, std::min(t, blocks));
  for (int i = 0; i < t; ++i) {
    const int b0 = (int)((int64_t)blocks * i / t), b1 = (int)((int64_t)blocks * (i + 1) / t);
    out.emplace_back(std::min(n, b0 * q), std::min(n, b1 * q));
  }
}

constexpr int PBUF_FLOATS = (SCRATCH_BYTES - PBUF_OFF) / 4;

// parts of a row of K <= 2048 values (the kernel's parts_of): the fewest of 1, 2, 4, 8 with at
// most 256 values each; equal parts of a multiple of 8 values
int row_parts(int64_t K) { return K <= 256 ? 1 : K <= 512 ? 2 : K <= 1024 ? 4 : 8; }
bool parts_ok(int64_t K) { return K >= 8 && K <= 2048 && K % (8 * row_parts(K)) == 0; }
// rows per stage for the row-dot engine: whole batches (a warp reduces eight row parts at once,
// so a batch is 64 / parts rows) when at least one fits
int engine_rows(int64_t K) {
  const int r = rows_per_stage(K * 2), batch = 64 / row_parts(K);
  return r >= batch ? (r / batch) * batch : r;
}

int max_range(const std::vector<std::pair<int, int>>& r) {
  int m = 0;
  for (const auto& x : r) m = std::max(m, x.second - x.first);
  return m;
}

int op_tasks_default(const MkHandle* h, int n_units, int min_units_per_task) {
  return std::max(1, std::min(h->num_ctas, n_units / std::max(1, min_units_per_task)));
}

}  // namespace

// A 2-D tensor map over a row-major BF16 cache tensor [rows, cols] (cols 512 or 64): boxes of 64
// columns x TC_RPS rows with the 128-byte swizzle, out-of-range rows read as zeros. The encoder is
// the driver's cuTensorMapEncodeTiled, reached through the runtime's entry-point query so the
// library links no driver library.
static int encode_rows_map(CUtensorMap* map, void* base, uint64_t cols, uint64_t rows) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
        q != cudaDriverEntryPointSuccess)
      return fail(MK_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)TC_RPS};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MK_EINVAL, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return MK_OK;
}

static int add_op_impl(MkHandle* h, const MkOp& in, int32_t* op_index) {
  OpDev od{};
  od.op = in;
  od.ksplit = 1;
  od.aux[0] = -1;
  od.aux[1] = 0;
  const int opi = (int)h->ops.size();
  std::vector<std::pair<int, int>> ranges;
  auto req = [&](bool ok, const char* what) { return ok ? 0 : fail(MK_EINVAL, std::string("op ") + std::to_string(opi) + ": " + what); };
  const int T = in.ntasks;
  switch (in.type) {
    case MK_OP_EMBED: {
      if (int e = req(in.ptr[MK_P_EMB_W] && in.ptr[MK_P_EMB_TOKENS] && in.ptr[MK_P_EMB_OUT], "embed: null pointer")) return e;
      if (int e = req(in.ip[MK_I_EMB_H] % 8 == 0, "embed: H % 8")) return e;
      ranges.emplace_back(0, 1);
      break;
    }
    case MK_OP_GEMV:
    case MK_OP_STREAM: {
      const bool gemv = in.type == MK_OP_GEMV;
      const int64_t N = gemv ? in.ip[MK_I_GEMV_N] : in.ip[MK_I_ST_ROWS];
      const int64_t K = gemv ? in.ip[MK_I_GEMV_K] : in.ip[MK_I_ST_K];
      if (int e = req(N > 0 && K > 0 && K % 8 == 0, "gemv: N, K > 0 and K % 8 == 0")) return e;
      if (gemv) {
        if (int e = req(in.ptr[MK_P_GEMV_X] && in.ptr[MK_P_GEMV_W] && in.ptr[MK_P_GEMV_OUT], "gemv: null pointer")) return e;
        if (int e = req(!(in.flags & MK_F_NORM) || in.ptr[MK_P_GEMV_WNORM], "gemv: NORM needs w_norm")) return e;
        if (int e = req(!(in.flags & MK_F_RESIDUAL) || in.ptr[MK_P_GEMV_RES], "gemv: RESIDUAL needs res")) return e;
        if (int e = req(!(in.flags & MK_F_ARGMAX) || in.ptr[MK_P_GEMV_TOKENS], "gemv: ARGMAX needs tokens")) return e;
        if (int e = req(!(in.flags & MK_F_NORM) || K * 2 <= XBUF_BYTES, "gemv: norm row exceeds the staging buffer")) return e;
      }
      if (K <= 2048) {
        od.ksplit = 1;
      } else {
        // one row per stage, the consumer warps share its K (parts of equal length, 16-byte
        // aligned, at most 2048 values each)
        od.ksplit = NUM_CONSUMER_WARPS;
        if (int e = req(K % (8 * NUM_CONSUMER_WARPS) == 0 && K / NUM_CONSUMER_WARPS <= 1536,
                        "gemv: K > 2048 must split into 8 parts of <= 1536, multiples of 8"))
          return e;
        if (int e = req(K * 2 <= STAGE_BYTES, "gemv: a K-split row must fit one stage")) return e;
        if (int e = req(!(in.flags & MK_F_ARGMAX), "gemv: ARGMAX with K-split unsupported")) return e;
      }
      od.rps = od.ksplit > 1 ? 1 : engine_rows(K);
      const int t = T > 0 ? T : op_tasks_default(h, (int)N, od.ksplit > 1 ? 1 : 8);
      split_even(ranges, (int)N, t);
      if (int e = req(od.ksplit > 1 || parts_ok(K), "gemv: K must split into equal parts of multiples of 8")) return e;
      const int parts = od.ksplit > 1 ? NUM_CONSUMER_WARPS : row_parts(K);
      if (int e = req(max_range(ranges) * parts <= PBUF_FLOATS, "gemv: rows per task exceed the partial buffer")) return e;
      break;
    }
    case MK_OP_MLA_PREP: {
      const int64_t NH = in.ip[MK_I_PREP_NH], DN = in.ip[MK_I_PREP_DN], DR = in.ip[MK_I_PREP_DR], DC = in.ip[MK_I_PREP_DC];
      for (int i = 0; i <= MK_P_PREP_QPE; ++i)
        if (int e = req(in.ptr[i] != nullptr, "prep: null pointer")) return e;
      if (int e = req(DN % 8 == 0 && DN <= 256 && DR % 2 == 0 && DC % 8 == 0 && DC * 2 <= XBUF_BYTES,
                      "prep: dims (DN % 8, DN <= 256, DR even, DC % 8)"))
        return e;
      const int64_t SMAX = in.ip[MK_I_PREP_SMAX];
      if (int e = req(SMAX >= 1, "prep: s_max >= 1")) return e;
      h->cache_rows = h->cache_rows > 0 ? std::min(h->cache_rows, SMAX) : SMAX;
      od.rps = engine_rows(DN);
      int t = T > 0 ? T : op_tasks_default(h, (int)(NH * DC), 16);
      t = std::max(t, (int)NH);       // at most DC rows, so a task touches at most two heads
      if (t > NH) {
        // task 0 writes the cache row (latent norm, RoPE) first: it takes no W_uk rows, so it
        // does not end after the others
        std::vector<std::pair<int, int>> rest;
        split_even(rest, (int)(NH * DC), t - 1);
        ranges.emplace_back(0, 0);
        ranges.insert(ranges.end(), rest.begin(), rest.end());
      } else {
        split_even(ranges, (int)(NH * DC), t);
      }
      if (int e = req(max_range(ranges) <= PBUF_FLOATS && max_range(ranges) <= DC,
                      "prep: rows per task exceed the partial buffer or one head"))
        return e;
      break;
    }
    case MK_OP_MLA_ATTEND: {
      const int64_t NH = in.ip[MK_I_ATT_NH], DC = in.ip[MK_I_ATT_DC], DR = in.ip[MK_I_ATT_DR];
      const int64_t S = in.ip[MK_I_ATT_SPLIT], HG = in.ip[MK_I_ATT_HGROUP], NS = in.ip[MK_I_ATT_NSPLITS];
      const bool tc = (in.flags & MK_F_TC) != 0;
      for (int i = 0; i <= MK_P_ATT_PARTIALS; ++i)
        if (int e = req(in.ptr[i] != nullptr, "attend: null pointer")) return e;
      if (int e = req(NS * S >= in.ip[MK_I_ATT_SMAX] && S >= 1, "attend: n_splits * split < s_max")) return e;
      if (int e = req(in.ip[MK_I_ATT_PROW] >= DC + 1 && in.ip[MK_I_ATT_PROW] % 4 == 0 &&
                          ((uintptr_t)in.ptr[MK_P_ATT_PARTIALS] & 15) == 0,
                      "attend: partials rows (>= DC + 1 floats, a multiple of 4, 16-byte aligned)"))
        return e;
      const int64_t QN = in.ip[MK_I_ATT_CPARTS] > 0 ? in.ip[MK_I_ATT_CPARTS] : 1;
      if (tc) {
        // the tensor-core form: all 16 heads of a split in one task (per latent-column part), rows
        // as TMA boxes of the caller's cache tensors (16-byte aligned bases; rows of 1,024 and 128 bytes)
        if (int e = req(QN == 1 || QN == 2 || QN == 4 || QN == 8, "attend TC: 1, 2, 4 or 8 column parts")) return e;
        if (int e = req(NH == 16 && DC == 512 && DR == 64 && HG == 16 && in.ip[MK_I_ATT_SMAX] >= 1 &&
                            in.ip[MK_I_ATT_SMAX] < (1 << 30) && ((uintptr_t)in.ptr[MK_P_ATT_CKV] & 15) == 0 &&
                            ((uintptr_t)in.ptr[MK_P_ATT_KPE] & 15) == 0,
                        "attend TC: 16 heads, DC 512, DR 64, head group 16, 16-byte aligned cache tensors"))
          return e;
      } else {
        if (int e = req(HG == 1 || (NH % HG == 0 && HG % 2 == 0 && DC == 512 && DR == 64),
                        "attend: head group 1, or an even group dividing the heads at DC 512, DR 64")) return e;
        // the general (non-512/64) path keeps at most 4 latent and 2 rope columns per lane
        if (int e = req(NH % HG == 0 && DC % 32 == 0 && DR % 2 == 0 &&
                            ((DC == 512 && DR == 64) || (DC <= 128 && (DR <= 32 || DR == 64))),
                        "attend: dims (DC 512 with DR 64, or DC <= 128 a multiple of 32 with DR even, <= 32 or 64)"))
          return e;
        const int rps = (int)(STAGE_BYTES / ((DC + DR) * 2));
        if (int e = req(div_up(S, rps) <= NSTAGES, "attend: a split must fit the ring")) return e;
        if (int e = req(S % 4 == 0 && 4096 + 2 * (((3 * S + 4) * 4 + S * 2 + 15) / 16 * 16) <= SCRATCH_BYTES &&
                            (DC + DR) * 2 <= 4096,
                        "attend: scores exceed scratch")) return e;
        od.rps = rps;
      }
      for (int64_t j = 0; j < NS; ++j)
        for (int64_t g = 0; g < (tc ? QN : NH / HG); ++g) ranges.emplace_back((int)g, (int)j);
      od.op.ip[MK_I_ATT_CPARTS] = tc ? QN : 1;
      od.aux[0] = -2;     // resolved at finalize: the chain's last operator, previous iteration
      od.aux[1] = 1;
      od.aux[2] = tc ? h->n_tc++ : -1;   // its pair of tensor maps
      break;
    }
    case MK_OP_MLA_MERGE_UV: {
      const int64_t NH = in.ip[MK_I_MRG_NH], DV = in.ip[MK_I_MRG_DV], DC = in.ip[MK_I_MRG_DC];
      for (int i = 0; i <= MK_P_MRG_OUT; ++i)
        if (int e = req(in.ptr[i] != nullptr, "merge: null pointer")) return e;
      if (int e = req(parts_ok(DC) && DC <= 1024, "merge: DC <= 1024 in equal parts of multiples of 8")) return e;
      if (int e = req(in.ip[MK_I_MRG_PROW] >= DC + 1 && in.ip[MK_I_MRG_PROW] % 4 == 0 &&
                          ((uintptr_t)in.ptr[MK_P_MRG_PARTIALS] & 15) == 0,
                      "merge: partials rows (>= DC + 1 floats, a multiple of 4, 16-byte aligned)"))
        return e;
      od.rps = engine_rows(DC);
      int t = T > 0 ? T : op_tasks_default(h, (int)(NH * DV), 8);
      t = std::max(t, (int)NH);       // a task spans at most two heads (one head's rows or fewer)
      split_even(ranges, (int)(NH * DV), t);
      for (auto& r : ranges)
        if (int e = req((r.second - 1) / DV - r.first / DV <= 1 || (r.second - r.first) <= DV, "merge: range")) return e;
      int maxh = 0;
      for (auto& r : ranges) maxh = std::max(maxh, (int)((r.second - 1) / DV - r.first / DV + 1));
      if (int e = req(maxh * DC * 2 <= XBUF_BYTES && maxh * DC <= 4 * NUM_CONSUMERS,
                      "merge: heads per task exceed the staging buffer"))
        return e;
      if (int e = req(max_range(ranges) * row_parts(DC) <= PBUF_FLOATS && maxh * (in.ip[MK_I_MRG_NSPLITS] + 1) <= PBUF_FLOATS,
                      "merge: rows or splits per task exceed the partial buffer"))
        return e;
      break;
    }
    case MK_OP_ROUTER: {
      const int64_t H = in.ip[MK_I_RT_H], E = in.ip[MK_I_RT_E], TOPK = in.ip[MK_I_RT_TOPK], NF = in.ip[MK_I_RT_NFORCED];
      for (int i = 0; i <= MK_P_RT_MASK; ++i)
        if (int e = req(in.ptr[i] != nullptr, "router: null pointer")) return e;
      if (int e = req(H % 8 == 0 && H <= 2048 && E >= 1 && E <= 256 && TOPK >= 1 && TOPK <= E &&
                          TOPK + NF <= MAX_ROUTED,
                      "router: dims (H <= 2048, E <= 256, TOPK + forced <= 16)"))
        return e;
      if (int e = req(((uintptr_t)in.ptr[MK_P_RT_LOGTAG] & 7) == 0 && ((uintptr_t)in.ptr[MK_P_RT_MASKTAG] & 7) == 0,
                      "router: 8-byte aligned tagged words"))
        return e;
      if (in.ptr[MK_P_RT_LOGTAG]) h->tagged.emplace_back(in.ptr[MK_P_RT_LOGTAG], (size_t)E * 8);
      if (in.ptr[MK_P_RT_MASKTAG]) h->tagged.emplace_back(in.ptr[MK_P_RT_MASKTAG], (size_t)(TOPK + NF) * 8);
      od.rps = engine_rows(H);
      const int t = T > 0 ? T : div_up(E, od.rps);
      split_even(ranges, (int)E, t);
      if (int e = req(parts_ok(H) && H * 2 <= XBUF_BYTES && max_range(ranges) * row_parts(H) <= PBUF_FLOATS,
                      "router: scratch (H in equal parts of multiples of 8)"))
        return e;
      break;
    }
    case MK_OP_GATEUP: {
      const int64_t K = in.ip[MK_I_GU_K], I = in.ip[MK_I_GU_I], G = in.ip[MK_I_GU_GROUPS];
      if (int e = req(in.ptr[MK_P_GU_X] && in.ptr[MK_P_GU_W] && in.ptr[MK_P_GU_ACT], "gateup: null pointer")) return e;
      if (int e = req(K % 8 == 0 && K <= 2048 && I > 0 && G >= 1, "gateup: dims (K % 8, K <= 2048)")) return e;
      if (int e = req(!(in.flags & MK_F_EXPERT) || (in.ptr[MK_P_GU_MASK] && in.ip[MK_I_GU_NEXP] > 0),
                      "gateup: EXPERT needs mask and n_experts"))
        return e;
      if (int e = req(!(in.flags & MK_F_NORM) || in.ptr[MK_P_GU_WNORM], "gateup: NORM needs w_norm")) return e;
      od.rps = std::max(2, engine_rows(K) & ~1);
      const int t = T > 0 ? T : op_tasks_default(h, (int)(G * I), 4);
      split_even(ranges, (int)(G * I), t);
      if (int e = req(parts_ok(K) && K * 2 <= XBUF_BYTES && max_range(ranges) * 2 * row_parts(K) <= PBUF_FLOATS,
                      "gateup: K parts, or pairs per task exceed the partial buffer"))
        return e;
      if (in.flags & MK_F_EP) {
        // the ranges are computed at run time over the owned slots; the host's are placeholders
        if (int e = req((in.flags & MK_F_EXPERT) && G <= MAX_ROUTED && in.ip[MK_I_GU_SLOT0] >= 0 &&
                            in.ip[MK_I_GU_SLOT0] + G <= MAX_ROUTED && in.ip[MK_I_GU_EPWORLD] >= 1 &&
                            in.ip[MK_I_GU_EPWORLD] <= MK_EP_MAX_RANKS && in.ip[MK_I_GU_EPRANK] >= 0 &&
                            in.ip[MK_I_GU_EPRANK] < in.ip[MK_I_GU_EPWORLD],
                        "gateup EP: experts, first slot + groups <= 16, a rank of at most 8"))
          return e;
      }
      if ((in.flags & MK_F_EXPERT) && !(in.flags & MK_F_STATIC_IDS))
        od.aux[0] = -3;   // resolved at finalize: the nearest router
      break;
    }
    case MK_OP_W2_COMBINE: {
      const int64_t H = in.ip[MK_I_W2_H], I = in.ip[MK_I_W2_I], NS = in.ip[MK_I_W2_SLOTS];
      for (int i = 0; i <= MK_P_W2_XRES; ++i)
        if (int e = req(in.ptr[i] != nullptr, "w2: null pointer")) return e;
      if (int e = req(parts_ok(I) && NS >= 1 && NS <= MAX_ROUTED && in.ip[MK_I_W2_NEXP] > 0,
                      "w2: dims (I in equal parts of multiples of 8, slots <= 16)"))
        return e;
      od.rps = engine_rows(I);
      const int t = T > 0 ? T : op_tasks_default(h, (int)H, 8);
      const bool ep = (in.flags & MK_F_EP) != 0;
      // expert parallelism exchanges 64-bit words of two rows: every task's rows start even
      split_even(ranges, (int)H, t, ep ? 2 : 1);
      if (ep) {
        if (int e = req(in.ptr[MK_P_W2_PEERS] && !in.ptr[MK_P_W2_OUT8] && H % 2 == 0 && in.ip[MK_I_W2_TOPK] >= 1 &&
                            in.ip[MK_I_W2_TOPK] <= NS && in.ip[MK_I_W2_EPWORLD] >= 1 &&
                            in.ip[MK_I_W2_EPWORLD] <= MK_EP_MAX_RANKS && in.ip[MK_I_W2_EPRANK] >= 0 &&
                            in.ip[MK_I_W2_EPRANK] < in.ip[MK_I_W2_EPWORLD] && in.ip[MK_I_W2_LAYER] >= 0 &&
                            (int)ranges.size() <= MK_EP_MAX_TASKS,
                        "w2 EP: peers (no out8), even H, topk, a rank of at most 8, at most 256 tasks"))
          return e;
      }
      if (int e = req(w2_aux_off((int)NS, (int)I) + w2_aux_bytes((int)NS, (int)max_range(ranges)) <= W2_PBUF_OFF &&
                          NS * max_range(ranges) * row_parts(I) * 4 <= SCRATCH_BYTES - W2_PBUF_OFF,
                      "w2: slots x I or rows per task exceed the scratch"))
        return e;
      od.aux[0] = -3;
      break;
    }
    case MK_OP_MOE_UNITS: {
      const int64_t H = in.ip[MK_I_MU_H], I = in.ip[MK_I_MU_I], S0 = in.ip[MK_I_MU_SLOT0], NSL = in.ip[MK_I_MU_NSLOTS];
      const int64_t NS = in.ip[MK_I_MU_NS], NE = in.ip[MK_I_MU_NEXP], F0 = in.ip[MK_I_MU_FIXED0];
      const bool fixed = (in.flags & MK_F_STATIC_IDS) != 0, routed = (in.flags & MK_F_EXPERT) != 0;
      if (int e = req(in.ptr[MK_P_MU_X] && in.ptr[MK_P_MU_W13] && in.ptr[MK_P_MU_W2F] && in.ptr[MK_P_MU_SUMS] &&
                          (!routed || in.ptr[MK_P_MU_MASK]),
                      "moe units: null pointer (x, W13, W2F, sums; mask with routed slots)"))
        return e;
      if (int e = req(!(in.flags & MK_F_NORM) || in.ptr[MK_P_MU_WNORM], "moe units: NORM needs w_norm")) return e;
      if (int e = req(parts_ok(H) && H * 2 <= XBUF_BYTES && parts_ok(I) && (I / unit_parts((int)I)) % 8 == 0,
                      "moe units: H and I in equal parts of multiples of 8 (H <= 2048)"))
        return e;
      if (int e = req(NSL >= 1 && S0 >= 0 && S0 + NSL <= NS && NS <= MAX_ROUTED && NE > 0 && F0 >= S0 &&
                          F0 <= S0 + NSL && (F0 == S0 + NSL || fixed) && (F0 == S0 || routed) &&
                          (!fixed || (in.ip[MK_I_MU_EXP0] >= 0 && in.ip[MK_I_MU_EXP0] + (S0 + NSL - F0) <= NE)),
                      "moe units: slots (SLOT0 <= FIXED0 <= SLOT0 + NSLOTS <= NS <= 16; STATIC_IDS for fixed "
                      "slots, EXPERT for routed ones) and experts"))
        return e;
      if (int e = req(((uintptr_t)in.ptr[MK_P_MU_W13] & 15) == 0 && ((uintptr_t)in.ptr[MK_P_MU_W2F] & 15) == 0 &&
                          ((uintptr_t)in.ptr[MK_P_MU_SUMS] & 15) == 0,
                      "moe units: 16-byte aligned W13, W2F and sums"))
        return e;
      if (int e = req(!(in.flags & MK_F_EP), "moe units: expert parallelism uses GATEUP and W2_COMBINE")) return e;
      if (int e = req(!(in.flags & MK_F_FP8) || (in.ptr[MK_P_MU_SCALE13] && H % 16 == 0 &&
                                                  ((uintptr_t)in.ptr[MK_P_MU_SCALE13] & 3) == 0),
                      "moe units: FP8 needs the gate/up scales and H a multiple of 16"))
        return e;
      if (int e = req(!in.ptr[MK_P_MU_MASKTAG] || (NE <= 256 && ((uintptr_t)in.ptr[MK_P_MU_MASKTAG] & 7) == 0),
                      "moe units: tagged slot experts need experts < 256 and 8-byte aligned words"))
        return e;
      // units u = ((s - SLOT0) KP + p) 8 + q with lanes (a unit's bytes are proportional to its lanes).
      // Each task gets a list: fixed-slot units, then routed-slot units, each kind placed longest
      // first onto the task with the least of that kind: the fixed units fill the time before the
      // router is done, and every task's routed units, which start together after it, end together.
      const int KP = unit_parts((int)I), l8 = (int)(I / KP) / 8;
      const int ur = (int)((F0 - S0) * KP * 8), U = (int)(NSL * KP * 8);
      if (int e = req(U < 65536, "moe units: too many units")) return e;
      int live = 0;
      for (int u = 0; u < U; ++u) live += unit_lanes(u & 7, l8) > 0;
      const int t = std::max(1, std::min(T > 0 ? T : h->num_ctas, live));
      const int64_t FT = in.ip[MK_I_MU_FTASKS];
      if (int e = req(FT >= 0, "moe units: FTASKS >= 0")) return e;
      // the tasks that share the fixed units (all of them when there are fewer tasks than FTASKS:
      // fewer live units than requested tasks)
      const int ft = FT > 0 ? std::min((int)FT, t) : t;
      std::vector<std::vector<uint16_t>> fl(t), rl(t);
      std::vector<int64_t> fload(t, 0), rload(t, 0);
      auto place = [&](int lo, int hi, bool fixed_kind) {
        std::vector<int> us;
        for (int u = lo; u < hi; ++u)
          if (unit_lanes(u & 7, l8) > 0) us.push_back(u);
        std::stable_sort(us.begin(), us.end(),
                         [&](int x, int y) { return unit_lanes(x & 7, l8) > unit_lanes(y & 7, l8); });
        std::vector<int64_t>& key = fixed_kind ? fload : rload;
        const int nt = fixed_kind ? ft : t;
        for (int u : us) {
          int k = 0;
          for (int j = 1; j < nt; ++j)
            if (key[j] < key[k]) k = j;
          (fixed_kind ? fl : rl)[k].push_back((uint16_t)u);
          key[k] += unit_lanes(u & 7, l8);
        }
      };
      place(ur, U, true);
      place(0, ur, false);
      for (int k = 0; k < t; ++k) {
        std::sort(fl[k].begin(), fl[k].end());
        std::sort(rl[k].begin(), rl[k].end());
        const int off = (int)h->units.size();
        h->units.insert(h->units.end(), fl[k].begin(), fl[k].end());
        h->units.insert(h->units.end(), rl[k].begin(), rl[k].end());
        if (int e = req(fl[k].size() < 65536 && rl[k].size() < 65536, "moe units: list")) return e;
        ranges.emplace_back(off, (int)(fl[k].size() | (rl[k].size() << 16)));
      }
      if (routed) od.aux[0] = -3;   // resolved at finalize: the nearest router
      break;
    }
    case MK_OP_MOE_COMBINE: {
      const int64_t H = in.ip[MK_I_MC_H], I = in.ip[MK_I_MC_I], NS = in.ip[MK_I_MC_NS];
      if (int e = req(in.ptr[MK_P_MC_SUMS] && in.ptr[MK_P_MC_TOPKW] && in.ptr[MK_P_MC_XRES], "moe combine: null pointer"))
        return e;
      if (int e = req(H >= 1 && parts_ok(I) && NS >= 1 && NS <= MAX_ROUTED, "moe combine: dims")) return e;
      if (int e = req(!(in.flags & MK_F_FP8) || (in.ptr[MK_P_MC_MASK] && in.ptr[MK_P_MC_SCALE2]),
                      "moe combine: FP8 needs the slots' experts and the down scales"))
        return e;
      const int t = T > 0 ? T : op_tasks_default(h, (int)H, 8);
      split_even(ranges, (int)H, t);
      const int KP = unit_parts((int)I);
      if (int e = req((NS * KP + NS + 1) * max_range(ranges) * 4 + 2 * MAX_ROUTED * 4 <= SCRATCH_BYTES,
                      "moe combine: rows per task exceed the scratch"))
        return e;
      break;
    }
    case MK_OP_COPY: {
      if (int e = req(in.ptr[MK_P_CP_SRC] && in.ptr[MK_P_CP_DST] && in.ip[MK_I_CP_N] > 0 && in.ip[MK_I_CP_N] % 8 == 0 &&
                          ((uintptr_t)in.ptr[MK_P_CP_SRC] & 15) == 0 && ((uintptr_t)in.ptr[MK_P_CP_DST] & 15) == 0,
                      "copy: 16-byte aligned pointers and n a multiple of 8"))
        return e;
      ranges.emplace_back(0, 1);
      break;
    }
    default:
      return fail(MK_EINVAL, "unknown operator type " + std::to_string(in.type));
  }
  od.ntasks = (int)ranges.size();
  od.task0 = (int)h->tasks.size();
  od.op.ntasks = od.ntasks;
  for (int i = 0; i < od.ntasks; ++i) h->tasks.push_back(TaskDev{opi, i, ranges[i].first, ranges[i].second});
  for (int j = 0; j < 2; ++j) { od.dep_op[j] = -1; od.dep_n[j] = 0; od.dep_lag[j] = 0; }
  h->ops.push_back(od);
  h->deps.emplace_back();
  if (op_index) *op_index = opi;
  return MK_OK;
}

static void free_device(MkHandle* h) {
  void* ptrs[] = {h->d_ops, h->d_cta_off, h->d_ctask, h->d_events, h->d_arrive,
                  h->d_status, h->d_amax_val, h->d_amax_idx, h->d_trace, h->d_trace_count, h->d_tmaps,
                  h->d_units};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  h->d_tmaps = nullptr;
  h->d_units = nullptr;
  h->d_ops = nullptr; h->d_cta_off = nullptr; h->d_ctask = nullptr;
  h->d_events = nullptr; h->d_arrive = nullptr; h->d_status = nullptr; h->d_amax_val = nullptr;
  h->d_amax_idx = nullptr; h->d_trace = nullptr; h->d_trace_count = nullptr;
}

extern "C" {

int mk_version(void) { return MK_ABI_VERSION; }

const char* mk_last_error(void) { return g_err.c_str(); }

int mk_create(const MkConfig* cfg, MkHandle** out) {
  if (!cfg || !out) return fail(MK_EINVAL, "mk_create: null argument");
  auto* h = new MkHandle();
  h->cfg = *cfg;
  if (h->cfg.wait_timeout_ns <= 0) h->cfg.wait_timeout_ns = 2000000000LL;
  cudaError_t e = cudaSetDevice(cfg->device);
  if (e != cudaSuccess) { delete h; return fail(MK_ECUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e)); }
  cudaDeviceProp prop{};
  e = cudaGetDeviceProperties(&prop, cfg->device);
  if (e != cudaSuccess) { delete h; return fail(MK_ECUDA, std::string("cudaGetDeviceProperties: ") + cudaGetErrorString(e)); }
  if (prop.major != 10) { delete h; return fail(MK_EINVAL, "device is not sm_100 (Blackwell B200)"); }
  h->num_sms = prop.multiProcessorCount;
  h->num_ctas = cfg->num_ctas > 0 ? std::min(cfg->num_ctas, h->num_sms) : h->num_sms;
  *out = h;
  return MK_OK;
}

int mk_add_op(MkHandle* h, const MkOp* op, int32_t* op_index) {
  if (!h || !op) return fail(MK_EINVAL, "mk_add_op: null argument");
  if (h->finalized) return fail(MK_ESTATE, "mk_add_op after mk_finalize");
  return add_op_impl(h, *op, op_index);
}

int mk_ep_alloc(int32_t device, size_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes == 0) return fail(MK_EINVAL, "mk_ep_alloc: bad argument");
  MK_CUDA(cudaSetDevice(device));
  MK_CUDA(cudaMalloc(dev_ptr, bytes));
  MK_CUDA(cudaMemset(*dev_ptr, 0, bytes));
  MK_CUDA(cudaDeviceSynchronize());
  return MK_OK;
}
int mk_ep_free(void* dev_ptr) {
  if (dev_ptr) MK_CUDA(cudaFree(dev_ptr));
  return MK_OK;
}
int mk_ep_ipc_handle(void* dev_ptr, void* handle64) {
  if (!dev_ptr || !handle64) return fail(MK_EINVAL, "mk_ep_ipc_handle: bad argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handles are 64 bytes");
  cudaIpcMemHandle_t hd;
  MK_CUDA(cudaIpcGetMemHandle(&hd, dev_ptr));
  std::memcpy(handle64, &hd, sizeof(hd));
  return MK_OK;
}
int mk_ep_ipc_open(int32_t device, const void* handle64, void** peer_ptr) {
  if (!handle64 || !peer_ptr) return fail(MK_EINVAL, "mk_ep_ipc_open: bad argument");
  cudaIpcMemHandle_t hd;
  std::memcpy(&hd, handle64, sizeof(hd));
  MK_CUDA(cudaSetDevice(device));
  MK_CUDA(cudaIpcOpenMemHandle(peer_ptr, hd, cudaIpcMemLazyEnablePeerAccess));
  return MK_OK;
}
int mk_ep_ipc_close(void* peer_ptr) {
  if (peer_ptr) MK_CUDA(cudaIpcCloseMemHandle(peer_ptr));
  return MK_OK;
}

int mk_set_op_deps(MkHandle* h, int32_t op_index, const int32_t* dep_ops, int32_t n) {
  if (!h || op_index < 0 || op_index >= (int)h->ops.size() || n < 1 || n > 2 || !dep_ops)
    return fail(MK_EINVAL, "mk_set_op_deps: bad argument (1 or 2 dependencies)");
  if (h->finalized) return fail(MK_ESTATE, "mk_set_op_deps after mk_finalize");
  std::vector<int32_t> d(dep_ops, dep_ops + n);
  for (int32_t x : d)
    if (x < 0 || x >= op_index) return fail(MK_EINVAL, "mk_set_op_deps: a dependency must be an earlier operator");
  if (n == 2 && d[0] == d[1]) return fail(MK_EINVAL, "mk_set_op_deps: duplicate dependency");
  h->deps[op_index] = d;
  return MK_OK;
}

int mk_op_tasks(MkHandle* h, int32_t op_index, int32_t* ntasks) {
  if (!h || !ntasks || op_index < 0 || op_index >= (int)h->ops.size()) return fail(MK_EINVAL, "mk_op_tasks: bad argument");
  *ntasks = h->ops[op_index].ntasks;
  return MK_OK;
}

int mk_finalize(MkHandle* h) {
  if (!h) return fail(MK_EINVAL, "mk_finalize: null handle");
  if (h->finalized) return fail(MK_ESTATE, "mk_finalize twice");
  if (h->ops.empty()) return fail(MK_EINVAL, "mk_finalize: no operators");
  const int nops = (int)h->ops.size();
  // producer-side dependencies
  for (int i = 0; i < nops; ++i) {
    OpDev& od = h->ops[i];
    if (od.aux[0] == -2) {            // cache rows: the nearest cache writer, previous iteration
      int w = nops - 1;
      for (int k = i - 1; k >= 0; --k)
        if (h->ops[k].op.type == MK_OP_MLA_PREP) { w = k; break; }
      od.aux[0] = w;
      od.aux[1] = 1;
    } else if (od.aux[0] == -3) {     // expert ids: the nearest router before this operator
      int r = -1;
      for (int k = i - 1; k >= 0; --k)
        if (h->ops[k].op.type == MK_OP_ROUTER) { r = k; break; }
      if (r < 0) return fail(MK_EINVAL, "op " + std::to_string(i) + ": routed experts without a router before them");
      od.aux[0] = r;
      od.aux[1] = 0;
    }
  }
  // expert parallelism: the exchange geometry the peer table was allocated for must hold this
  // operator's (a mismatch would make the kernel store past the end of a peer's buffer)
  for (int i = 0; i < nops; ++i) {
    const OpDev& od = h->ops[i];
    if (od.op.type != MK_OP_W2_COMBINE || !(od.op.flags & MK_F_EP)) continue;
    MkEpPeers pe{};
    MK_CUDA(cudaSetDevice(h->cfg.device));
    MK_CUDA(cudaMemcpy(&pe, od.op.ptr[MK_P_W2_PEERS], sizeof(pe), cudaMemcpyDeviceToHost));
    bool ok = pe.nranks == od.op.ip[MK_I_W2_EPWORLD] && pe.rank == od.op.ip[MK_I_W2_EPRANK] &&
              pe.n_slots == od.op.ip[MK_I_W2_SLOTS] && pe.hidden == od.op.ip[MK_I_W2_H] &&
              od.op.ip[MK_I_W2_LAYER] < pe.n_layers;
    for (int r = 0; ok && r < pe.nranks; ++r) ok = pe.xch[r] != nullptr;
    if (!ok)
      return fail(MK_EINVAL, "op " + std::to_string(i) + ": the expert-parallel peer table (ranks " +
                                 std::to_string(pe.nranks) + ", rank " + std::to_string(pe.rank) + ", layers " +
                                 std::to_string(pe.n_layers) + ", slots " + std::to_string(pe.n_slots) + ", hidden " +
                                 std::to_string(pe.hidden) + ") does not match the operator");
  }
  // consumer-side dependencies: the previous operator unless set explicitly. The first operator
  // waits for the previous iteration's sinks (the operators nothing else waits for, at most two),
  // so an iteration starts only when every operator of the one before is done.
  std::vector<char> has_dependent(nops, 0);
  for (int i = 1; i < nops; ++i) {
    OpDev& od = h->ops[i];
    std::vector<int32_t> d = h->deps[i];
    if (d.empty()) d.push_back(i - 1);
    for (int j = 0; j < 2; ++j) { od.dep_op[j] = -1; od.dep_n[j] = 0; od.dep_lag[j] = 0; }
    for (size_t j = 0; j < d.size(); ++j) {
      od.dep_op[j] = d[j]; od.dep_n[j] = h->ops[d[j]].ntasks; od.dep_lag[j] = 0;
      has_dependent[d[j]] = 1;
    }
  }
  {
    OpDev& od0 = h->ops[0];
    for (int j = 0; j < 2; ++j) { od0.dep_op[j] = -1; od0.dep_n[j] = 0; od0.dep_lag[j] = 0; }
    int n = 0;
    for (int i = nops - 1; i >= 0; --i) {
      if (has_dependent[i]) continue;
      if (n == 2) return fail(MK_EINVAL, "more than two operators end the chain (nothing waits for them)");
      od0.dep_op[n] = i; od0.dep_n[n] = h->ops[i].ntasks; od0.dep_lag[n] = 1;
      ++n;
    }
  }
  // deal tasks to CTAs in chain order: an operator with one task per CTA maps task t to CTA t;
  // smaller operators start at a rotating CTA so the extra work spreads
  h->cta_tasks.assign(h->num_ctas, {});
  int maxtasks = 1;
  for (int i = 0; i < nops; ++i) {
    const OpDev& od = h->ops[i];
    maxtasks = std::max(maxtasks, od.ntasks);
    // (expert units: always from the rotating start, so that tasks past FTASKS, dealt last, land on
    // the CTAs of the operators it runs beside)
    const bool units = od.op.type == MK_OP_MOE_UNITS;
    const int start = od.ntasks >= h->num_ctas && !units ? 0 : h->rr;
    for (int t = 0; t < od.ntasks; ++t) h->cta_tasks[(start + t) % h->num_ctas].push_back((uint32_t)(od.task0 + t));
    if (od.ntasks < h->num_ctas || units) h->rr = (h->rr + od.ntasks) % h->num_ctas;
  }
  std::vector<uint32_t> off(h->num_ctas + 1, 0);
  std::vector<CtaTask> list;
  for (int c = 0; c < h->num_ctas; ++c) {
    off[c] = (uint32_t)list.size();
    const auto& ct = h->cta_tasks[c];
    int run = 0;   // tasks of the same operator just before this one on this CTA
    for (size_t k = 0; k < ct.size(); ++k) {
      CtaTask e{};
      e.t = h->tasks[ct[k]];
      e.next_op = h->tasks[ct[(k + 1) % ct.size()]].op;
      // a run of one operator's tasks signals once, at its last task, for the whole run
      ++run;
      const bool last_of_run = k + 1 == ct.size() || e.next_op != e.t.op;
      e.signal = last_of_run ? run : 0;
      if (last_of_run) run = 0;
      list.push_back(e);
    }
  }
  off[h->num_ctas] = (uint32_t)list.size();
  MK_CUDA(cudaSetDevice(h->cfg.device));
  if (h->n_tc > 0) {
    std::vector<CUtensorMap> maps(2 * (size_t)h->n_tc);
    for (const OpDev& od : h->ops) {
      if (od.op.type != MK_OP_MLA_ATTEND || !(od.op.flags & MK_F_TC)) continue;
      const uint64_t smax = (uint64_t)od.op.ip[MK_I_ATT_SMAX];
      if (int e = encode_rows_map(&maps[2 * (size_t)od.aux[2]], od.op.ptr[MK_P_ATT_CKV], 512, smax)) return e;
      if (int e = encode_rows_map(&maps[2 * (size_t)od.aux[2] + 1], od.op.ptr[MK_P_ATT_KPE], 64, smax)) return e;
    }
    MK_CUDA(cudaMalloc(&h->d_tmaps, sizeof(CUtensorMap) * maps.size()));
    MK_CUDA(cudaMemcpy(h->d_tmaps, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice));
  }
  if (!h->units.empty()) {
    MK_CUDA(cudaMalloc(&h->d_units, sizeof(uint16_t) * h->units.size()));
    MK_CUDA(cudaMemcpy(h->d_units, h->units.data(), sizeof(uint16_t) * h->units.size(), cudaMemcpyHostToDevice));
  }
  MK_CUDA(cudaMalloc(&h->d_ops, sizeof(OpDev) * nops));
  MK_CUDA(cudaMalloc(&h->d_cta_off, sizeof(uint32_t) * off.size()));
  MK_CUDA(cudaMalloc(&h->d_ctask, sizeof(CtaTask) * std::max<size_t>(1, list.size())));
  MK_CUDA(cudaMalloc(&h->d_events, sizeof(uint32_t) * nops));
  MK_CUDA(cudaMalloc(&h->d_arrive, sizeof(uint32_t) * nops));
  MK_CUDA(cudaMalloc(&h->d_status, sizeof(DevStatus)));
  MK_CUDA(cudaMalloc(&h->d_amax_val, sizeof(float) * maxtasks));
  MK_CUDA(cudaMalloc(&h->d_amax_idx, sizeof(int32_t) * maxtasks));
  MK_CUDA(cudaMalloc(&h->d_trace_count, sizeof(uint32_t)));
  MK_CUDA(cudaMemcpy(h->d_ops, h->ops.data(), sizeof(OpDev) * nops, cudaMemcpyHostToDevice));
  MK_CUDA(cudaMemcpy(h->d_cta_off, off.data(), sizeof(uint32_t) * off.size(), cudaMemcpyHostToDevice));
  if (!list.empty())
    MK_CUDA(cudaMemcpy(h->d_ctask, list.data(), sizeof(CtaTask) * list.size(), cudaMemcpyHostToDevice));
  MK_CUDA(cudaMemset(h->d_events, 0, sizeof(uint32_t) * nops));
  MK_CUDA(cudaMemset(h->d_arrive, 0, sizeof(uint32_t) * nops));
  MK_CUDA(cudaMemset(h->d_status, 0, sizeof(DevStatus)));
  MK_CUDA(cudaMemset(h->d_trace_count, 0, sizeof(uint32_t)));
  if (h->cfg.trace) {
    h->trace_cap = (uint32_t)std::min<size_t>(h->tasks.size() * 64, 1u << 22);
    MK_CUDA(cudaMalloc(&h->d_trace, sizeof(MkTraceRecord) * h->trace_cap));
  }
  bool long_ctx = false, tc = false;
  for (const OpDev& od : h->ops) {
    if (od.op.type != MK_OP_MLA_ATTEND) continue;
    if (od.op.flags & MK_F_TC) tc = true;
    else if (od.op.ip[MK_I_ATT_HGROUP] > 1) long_ctx = true;
  }
  if (tc && long_ctx)
    return fail(MK_EINVAL, "one handle cannot mix the tensor-core attention with exact head groups > 1");
  h->variant = tc ? KV_TC : long_ctx ? KV_LONG : KV_SHORT;
  const auto kern = h->variant == KV_TC ? mk_persistent_kernel<KV_TC>
                    : h->variant == KV_LONG ? mk_persistent_kernel<KV_LONG> : mk_persistent_kernel<KV_SHORT>;
  MK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem)));
  int per_sm = 0;
  MK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NUM_THREADS, sizeof(Smem)));
  if (per_sm < 1) return fail(MK_EINVAL, "the persistent kernel does not fit an SM");
  h->gen = 1;
  for (const auto& tw : h->tagged) MK_CUDA(cudaMemset(tw.first, 0, tw.second));
  MK_CUDA(cudaDeviceSynchronize());
  h->finalized = true;
  return MK_OK;
}

int mk_launch(MkHandle* h, void* stream, int32_t iters, int32_t step, int32_t* meta_step) {
  if (!h) return fail(MK_EINVAL, "mk_launch: null handle");
  if (!h->finalized) return fail(MK_ESTATE, "mk_launch before mk_finalize");
  if (iters < 1) return fail(MK_EINVAL, "mk_launch: iters < 1");
  // iteration i appends cache row step + 1 + i and writes tokens[step + 2 + i]: both in the rows
  if (step < -1 || (h->cache_rows > 0 && (int64_t)step + 1 + iters >= h->cache_rows))
    return fail(MK_EINVAL, "mk_launch: positions step + 1 .. step + iters + 1 must lie in [0, s_max) (step " +
                               std::to_string(step) + ", iters " + std::to_string(iters) + ", s_max " +
                               std::to_string(h->cache_rows) + ")");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  MK_CUDA(cudaSetDevice(h->cfg.device));
  // the counters are 32-bit and grow by ntasks per iteration: restart them long before they wrap
  int maxtasks = 1;
  for (const auto& od : h->ops) maxtasks = std::max(maxtasks, od.ntasks);
  if ((h->gen + (uint64_t)iters) * (uint64_t)maxtasks >= (1ull << 31)) {
    MK_CUDA(cudaMemsetAsync(h->d_events, 0, sizeof(uint32_t) * h->ops.size(), s));
    MK_CUDA(cudaMemsetAsync(h->d_arrive, 0, sizeof(uint32_t) * h->ops.size(), s));
    for (const auto& tw : h->tagged) MK_CUDA(cudaMemsetAsync(tw.first, 0, tw.second, s));
    h->gen = 1;
  }
  if (h->d_trace) MK_CUDA(cudaMemsetAsync(h->d_trace_count, 0, sizeof(uint32_t), s));
  KernelParams P{};
  P.ops = h->d_ops;
  P.cta_off = h->d_cta_off;
  P.ctask = h->d_ctask;
  P.events = h->d_events;
  P.arrive = h->d_arrive;
  P.status = h->d_status;
  P.amax_val = h->d_amax_val;
  P.amax_idx = h->d_amax_idx;
  P.trace = h->d_trace;
  P.trace_count = h->d_trace_count;
  P.trace_cap = h->trace_cap;
  P.nops = (int32_t)h->ops.size();
  P.iters = iters;
  P.step = step;
  P.gen0 = (uint32_t)h->gen;
  P.block_op = h->block_op;
  P.timeout_ns = h->cfg.wait_timeout_ns;
  P.meta_step = meta_step;
  P.ep_gen0 = h->ep_gen;
  P.tmaps = h->d_tmaps;
  P.units = h->d_units;
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3((unsigned)h->num_ctas);
  lc.blockDim = dim3((unsigned)NUM_THREADS);
  lc.dynamicSmemBytes = sizeof(Smem);
  lc.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  if (h->variant == KV_TC) MK_CUDA(cudaLaunchKernelEx(&lc, mk_persistent_kernel<KV_TC>, P));
  else if (h->variant == KV_LONG) MK_CUDA(cudaLaunchKernelEx(&lc, mk_persistent_kernel<KV_LONG>, P));
  else MK_CUDA(cudaLaunchKernelEx(&lc, mk_persistent_kernel<KV_SHORT>, P));
  h->block_op = -1;
  h->gen += (uint64_t)iters;
  h->ep_gen += (uint32_t)iters;   // consumed even if the launch fails: every rank's tags stay equal
  h->launches++;
  h->last_stream = s;
  return MK_OK;
}

int mk_decode_token(MkHandle* h, void* stream, int64_t* tokens, int32_t step, const int64_t* token_in,
                    int64_t* token_out, int32_t* meta_step) {
  if (!h || !tokens || !token_in || !token_out) return fail(MK_EINVAL, "mk_decode_token: null argument");
  if (!h->finalized) return fail(MK_ESTATE, "mk_decode_token before mk_finalize");
  if (step < -1 || (h->cache_rows > 0 && (int64_t)step + 2 >= h->cache_rows))
    return fail(MK_EINVAL, "mk_decode_token: step + 2 must lie below s_max");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  MK_CUDA(cudaSetDevice(h->cfg.device));
  MK_CUDA(cudaMemcpyAsync(tokens + (step + 1), token_in, sizeof(int64_t), cudaMemcpyHostToDevice, s));
  if (int e = mk_launch(h, stream, 1, step, meta_step)) return e;
  MK_CUDA(cudaMemcpyAsync(token_out, tokens + (step + 2), sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  MK_CUDA(cudaStreamSynchronize(s));
  return MK_OK;
}

int mk_status(MkHandle* h, MkStatus* out) {
  if (!h || !out) return fail(MK_EINVAL, "mk_status: null argument");
  if (!h->finalized) return fail(MK_ESTATE, "mk_status before mk_finalize");
  MK_CUDA(cudaSetDevice(h->cfg.device));
  MK_CUDA(cudaStreamSynchronize(h->last_stream));
  DevStatus ds{};
  MK_CUDA(cudaMemcpy(&ds, h->d_status, sizeof(DevStatus), cudaMemcpyDeviceToHost));
  std::memset(out, 0, sizeof(*out));
  out->error = ds.error;
  out->err_op = ds.err_op;
  out->err_task = ds.err_task;
  out->err_cta = ds.err_cta;
  out->err_info = ds.err_info;
  out->aborted_ctas = ds.aborted_ctas;
  out->launches = h->launches;
  out->generation = h->gen - 1;
  if (ds.error) return fail(MK_EDEVICE, "device status error " + std::to_string(ds.error) + " at op " +
                                            std::to_string(ds.err_op) + " task " + std::to_string(ds.err_task));
  return MK_OK;
}

int mk_reset(MkHandle* h) {
  if (!h || !h->finalized) return fail(MK_ESTATE, "mk_reset: not finalized");
  MK_CUDA(cudaSetDevice(h->cfg.device));
  MK_CUDA(cudaStreamSynchronize(h->last_stream));
  MK_CUDA(cudaMemset(h->d_events, 0, sizeof(uint32_t) * h->ops.size()));
  MK_CUDA(cudaMemset(h->d_arrive, 0, sizeof(uint32_t) * h->ops.size()));
  MK_CUDA(cudaMemset(h->d_status, 0, sizeof(DevStatus)));
  for (const auto& tw : h->tagged) MK_CUDA(cudaMemset(tw.first, 0, tw.second));
  h->gen = 1;
  return MK_OK;
}

int mk_trace(MkHandle* h, MkTraceRecord* out, int64_t cap, int64_t* n) {
  if (!h || !n) return fail(MK_EINVAL, "mk_trace: null argument");
  if (!h->d_trace) return fail(MK_ESTATE, "mk_trace: the handle was created without trace");
  MK_CUDA(cudaSetDevice(h->cfg.device));
  MK_CUDA(cudaStreamSynchronize(h->last_stream));
  uint32_t cnt = 0;
  MK_CUDA(cudaMemcpy(&cnt, h->d_trace_count, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  const int64_t m = std::min<int64_t>(std::min<int64_t>(cnt, h->trace_cap), cap);
  if (out && m > 0) MK_CUDA(cudaMemcpy(out, h->d_trace, sizeof(MkTraceRecord) * m, cudaMemcpyDeviceToHost));
  *n = std::min<int64_t>(cnt, h->trace_cap);
  return MK_OK;
}

int mk_debug_block_op(MkHandle* h, int32_t op_index) {
  if (!h || op_index < 0 || op_index >= (int)h->ops.size()) return fail(MK_EINVAL, "mk_debug_block_op: bad argument");
  h->block_op = op_index;
  return MK_OK;
}

int mk_destroy(MkHandle* h) {
  if (!h) return MK_OK;
  cudaSetDevice(h->cfg.device);
  if (h->finalized) cudaStreamSynchronize(h->last_stream);
  free_device(h);
  delete h;
  return MK_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// self-test kernels of the deterministic arithmetic (bit-compared with oracle/detmath.py)

namespace {
__global__ void selftest_kernel(int fn, const void* x, void* out, int64_t n) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  switch (fn) {
    case 0: reinterpret_cast<float*>(out)[i] = det_exp(reinterpret_cast<const float*>(x)[i]); break;
    case 1: reinterpret_cast<float*>(out)[i] = det_log(reinterpret_cast<const float*>(x)[i]); break;
    case 2: reinterpret_cast<float*>(out)[i] = det_silu(reinterpret_cast<const float*>(x)[i]); break;
    case 3: reinterpret_cast<uint16_t*>(out)[i] = (uint16_t)f64_to_bf16_bits(reinterpret_cast<const double*>(x)[i]); break;
    case 4: reinterpret_cast<uint16_t*>(out)[i] = (uint16_t)f32_to_bf16_bits(reinterpret_cast<const float*>(x)[i]); break;
    default: break;
  }
}
}  // namespace

extern "C" int mk_selftest_math(int32_t fn, const void* x, void* out, int64_t n, void* stream) {
  if (fn < 0 || fn > 4 || !x || !out || n < 0) return fail(MK_EINVAL, "mk_selftest_math: bad argument");
  if (n == 0) return MK_OK;
  const int bs = 256;
  selftest_kernel<<<(unsigned)((n + bs - 1) / bs), bs, 0, reinterpret_cast<cudaStream_t>(stream)>>>(fn, x, out, n);
  MK_CUDA(cudaGetLastError());
  return MK_OK;
}
