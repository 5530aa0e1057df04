// mk_kernel.cuh -- the persistent decode kernel: one CTA per SM, eight consumer warps and one
// producer warp, walking a per-CTA task list that the host built from the operator chain.
//
// Scheduling (the reference's runtime, docs/fleet/03-runtime.md:1-90, resolved at build time):
// every operator has a completion counter in device memory; a task waits (bounded spin, acquire)
// until the previous operator's counter reaches its task count times the iteration's
// generation, runs, and adds one (release). Counters never reset inside a launch, so a whole
// greedy decode of `iters` tokens runs in one launch (D22 of the reference).
//
// Weight streaming: the producer warp walks the same task list ahead of the consumers and
// issues cp.async.bulk copies of each task's weight rows into a 6 x 32 KB ring (mbarrier full /
// empty pairs). Weights do not depend on activations, so the ring fills while the consumers
// still wait for the previous operator: only routed-expert weights wait for the router (their
// addresses), and latent-cache rows wait for the previous iteration.
#pragma once
#include "mk_ops.cuh"

namespace mk {

// Tensor-core attention (MK_F_TC) stage geometry, shared by the producer and attend_tc.
constexpr int TC_RPS = 24;                       // cache rows per stage
constexpr int TC_BOX = TC_RPS * 128;             // one 64-column box of a stage (1024-byte multiple)
constexpr int TC_STAGE_TX = 9 * TC_BOX;          // 8 latent boxes + 1 rope box
constexpr int TC_CHUNK_STAGES = 4;
constexpr int TC_CHUNK = TC_RPS * TC_CHUNK_STAGES;
constexpr int TC_QSTRIDE = 1168;                 // a head's 576 BF16 of Q + 16 bytes (rows shift banks)
constexpr int TC_PSTRIDE = (TC_CHUNK + 8) * 2;   // a head's chunk of P + 16 bytes
constexpr int TC_Q_OFF = 0;
constexpr int TC_P_OFF = TC_Q_OFF + 16 * TC_QSTRIDE;
constexpr int TC_OWN_OFF = TC_P_OFF + 16 * TC_PSTRIDE;
constexpr int TC_ZERO_OFF = TC_OWN_OFF + 576 * 2;
constexpr int TC_RED_OFF = TC_ZERO_OFF + 16;
constexpr int TC_HALF_OFF = TC_RED_OFF + 2 * NUM_CONSUMER_WARPS * 16 * 4;   // [4 pairs][32 lanes][8] partial scores
constexpr int TC_SCRATCH_END = TC_HALF_OFF + 4 * 32 * 8 * 4;
static_assert(TC_SCRATCH_END <= SCRATCH_BYTES, "tensor-core attention scratch");
static_assert(TC_STAGE_TX <= STAGE_BYTES && TC_CHUNK_STAGES < NSTAGES, "tensor-core attention stages");


// =============================================================================================
// producer
// =============================================================================================

struct Prod {
  uint32_t p_it;
};

__device__ __forceinline__ bool issue_stage(const KernelParams& P, Smem& sm, Prod& pr, const void* s0, uint32_t b0,
                                            const void* s1, uint32_t b1, uint32_t off1, uint32_t op, uint32_t task,
                                            int32_t aux = 0) {
  const uint32_t st = pr.p_it % NSTAGES, ph = (pr.p_it / NSTAGES) & 1u;
  if (!ring_wait(P, sm, &sm.empty[st], ph ^ 1u)) {
    report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_RING_TIMEOUT, op,
                 task, 2);
    return false;
  }
  sm.stage_aux[st] = aux;   // released to the stage's consumer by the arrive below
  mbar_arrive_expect_tx(&sm.full[st], b0 + b1);
  bulk_g2s(sm.ring[st], s0, b0, &sm.full[st]);
  if (b1) bulk_g2s(sm.ring[st] + off1, s1, b1, &sm.full[st]);
  pr.p_it++;
  return true;
}

// One stage of tensor-core attention rows: the 8 latent boxes and the rope box of rows [y, y + 24)
// (rows past the tensor's end arrive as zeros; the consumer never reads rows past its split).
__device__ __forceinline__ bool issue_stage_tma(const KernelParams& P, Smem& sm, Prod& pr, const void* tmap_c,
                                                const void* tmap_k, int y, uint32_t op, uint32_t task) {
  const uint32_t st = pr.p_it % NSTAGES, ph = (pr.p_it / NSTAGES) & 1u;
  if (!ring_wait(P, sm, &sm.empty[st], ph ^ 1u)) {
    report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_RING_TIMEOUT, op,
                 task, 2);
    return false;
  }
  mbar_arrive_expect_tx(&sm.full[st], (uint32_t)TC_STAGE_TX);
#pragma unroll 1
  for (int b = 0; b < 8; ++b) tma_load_2d(sm.ring[st] + b * TC_BOX, tmap_c, 64 * b, y, &sm.full[st]);
  tma_load_2d(sm.ring[st] + 8 * TC_BOX, tmap_k, 0, y, &sm.full[st]);
  pr.p_it++;
  return true;
}

// Streams every stage of one task. Returns false on an error (already reported).
__device__ bool produce_task(const KernelParams& P, Smem& sm, Prod& pr, const OpDev& od, const TaskDev& t,
                             const Iter& itx) {
  const uint32_t op = (uint32_t)t.op, task = (uint32_t)t.idx;
  const int type = od.op.type;
  // producer-side dependency: the router of this iteration (expert ids) or the previous
  // iteration (cache rows)
  if (od.aux[0] >= 0 && (type == MK_OP_GATEUP || type == MK_OP_W2_COMBINE || type == MK_OP_MLA_ATTEND)) {
    bool need = true;
    if (type == MK_OP_MLA_ATTEND) need = att_split(od, t, itx.pos).n_str > 0;
    if (need) {
      const OpDev& dep = P.ops[od.aux[0]];
      const uint32_t target = (uint32_t)dep.ntasks * (itx.g - (uint32_t)od.aux[1]);
      if (!wait_event(P, sm, &P.events[od.aux[0]], target, false)) {
        report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_WAIT_TIMEOUT,
                     op, task, 0x10000u | (uint32_t)od.aux[0]);
        return false;
      }
      fence_proxy_async_global();
    }
  }
  switch (type) {
    case MK_OP_GEMV:
    case MK_OP_MLA_PREP:
    case MK_OP_MLA_MERGE_UV:
    case MK_OP_ROUTER:
    case MK_OP_STREAM: {
      int K;
      const uint8_t* W;
      if (type == MK_OP_GEMV) { K = (int)I_(od, MK_I_GEMV_K); W = P_<const uint8_t>(od, MK_P_GEMV_W); }
      else if (type == MK_OP_MLA_PREP) { K = (int)I_(od, MK_I_PREP_DN); W = P_<const uint8_t>(od, MK_P_PREP_WUKT); }
      else if (type == MK_OP_MLA_MERGE_UV) { K = (int)I_(od, MK_I_MRG_DC); W = P_<const uint8_t>(od, MK_P_MRG_WUV); }
      else if (type == MK_OP_ROUTER) { K = (int)I_(od, MK_I_RT_H); W = P_<const uint8_t>(od, MK_P_RT_WGATE); }
      else { K = (int)I_(od, MK_I_ST_K); W = P_<const uint8_t>(od, MK_P_ST_W); }
      const size_t rb = (size_t)K * 2;
      for (int r = t.a; r < t.b; r += od.rps) {
        const int nr = min(od.rps, t.b - r);
        if (!issue_stage(P, sm, pr, W + (size_t)r * rb, (uint32_t)(nr * rb), nullptr, 0, 0, op, task)) return false;
      }
      return true;
    }
    case MK_OP_GATEUP: {
      const int K = (int)I_(od, MK_I_GU_K);
      const size_t rb = (size_t)K * 2;
      const uint8_t* W = P_<const uint8_t>(od, MK_P_GU_W);
      const bool expert = (od.op.flags & MK_F_EXPERT) != 0;
      const int32_t* mask = P_<const int32_t>(od, MK_P_GU_MASK);
      const int64_t estride = I_(od, MK_I_GU_ESTRIDE);
      const int nexp = (int)I_(od, MK_I_GU_NEXP);
      const GuMap gm = gu_map(od, t);
      int p = gm.a;
      GuChunk ch;
      while (gu_next(od, p, gm.b, ch)) {
        int e = 0;
        if (expert) {
          e = __ldcg(mask + gu_slot(gm, ch.group));
          if (e < 0 || e >= nexp) { report_error(P, sm, MK_DERR_BAD_EXPERT, op, task, (uint32_t)e); return false; }
        }
        const uint8_t* src = W + ((size_t)e * (size_t)estride + (size_t)ch.q * 2 * K) * 2;
        if (!issue_stage(P, sm, pr, src, (uint32_t)(2 * ch.np * rb), nullptr, 0, 0, op, task)) return false;
      }
      return true;
    }
    case MK_OP_W2_COMBINE: {
      const int H = (int)I_(od, MK_I_W2_H), I = (int)I_(od, MK_I_W2_I), NS = (int)I_(od, MK_I_W2_SLOTS);
      const size_t rb = (size_t)I * 2;
      const uint8_t* W = P_<const uint8_t>(od, MK_P_W2_W);
      const int32_t* mask = P_<const int32_t>(od, MK_P_W2_MASK);
      const int64_t estride = I_(od, MK_I_W2_ESTRIDE);
      const int nexp = (int)I_(od, MK_I_W2_NEXP);
      (void)H;
      (void)NS;
      for (uint32_t sl = w2_slots(od); sl; sl &= sl - 1u) {
        const int e = __ldcg(mask + (__ffs(sl) - 1));
        if (e < 0 || e >= nexp) { report_error(P, sm, MK_DERR_BAD_EXPERT, op, task, (uint32_t)e); return false; }
        const uint8_t* base = W + (size_t)e * (size_t)estride * 2;
        for (int r = t.a; r < t.b; r += od.rps) {
          const int nr = min(od.rps, t.b - r);
          if (!issue_stage(P, sm, pr, base + (size_t)r * rb, (uint32_t)(nr * rb), nullptr, 0, 0, op, task))
            return false;
        }
      }
      return true;
    }
    case MK_OP_MOE_UNITS: {
      // per unit: its lanes' gate/up rows (16 per lane: intermediates 8 l .. 8 l + 7 of the part,
      // gate and up interleaved), then its rows of the regrouped down projection. The fixed
      // slots' units first; the routed slots' units once the router has written the expert ids.
      const int H = (int)I_(od, MK_I_MU_H), I = (int)I_(od, MK_I_MU_I);
      const int KP = unit_parts(I), Lp = I / KP, l8 = Lp / 8, slot0 = (int)I_(od, MK_I_MU_SLOT0);
      const size_t eb = (od.op.flags & MK_F_FP8) ? 1 : 2;   // bytes per weight
      const int fixed0 = (int)I_(od, MK_I_MU_FIXED0), nexp = (int)I_(od, MK_I_MU_NEXP);
      const int r13 = unit_w13_rows((int64_t)H * (int64_t)eb);
      const uint8_t* W13 = P_<const uint8_t>(od, MK_P_MU_W13);
      const uint8_t* W2F = P_<const uint8_t>(od, MK_P_MU_W2F);
      const int32_t* mask = P_<const int32_t>(od, MK_P_MU_MASK);
      const uint64_t* mtag = P_<const uint64_t>(od, MK_P_MU_MASKTAG);
      uint64_t rexp_lo = 0u, rexp_hi = 0u;   // with mtag: the routed slots' experts, 8 bits per slot
      const MuList ml = mu_list(t);
      for (int v = 0; v < ml.nf + ml.nr; ++v) {
        if (v == ml.nf && mtag) {   // the first routed unit: every routed slot's tagged expert
          // eight slots' words in flight at a time (the router writes them together), again until
          // every word carries this iteration's tag
          const uint64_t t0 = globaltimer();
          for (int g0 = slot0; g0 < fixed0; g0 += 8) {
            const int ng = min(8, fixed0 - g0);
            uint32_t need = (1u << ng) - 1u;
            for (uint32_t n = 0; need; ++n) {
              uint64_t w[8];
#pragma unroll
              for (int k = 0; k < 8; ++k) w[k] = (need >> k) & 1u ? ld_relaxed_gpu_u64(mtag + g0 + k) : 0u;
#pragma unroll
              for (int k = 0; k < 8; ++k)
                if (((need >> k) & 1u) && (uint32_t)(w[k] >> 32) == itx.g) {
                  const int sl = g0 + k;
                  const uint64_t b = (uint64_t)((uint32_t)w[k] & 0xFFu) << (8 * ((sl - slot0) & 7));
                  if (sl - slot0 < 8) rexp_lo |= b;
                  else rexp_hi |= b;
                  need &= ~(1u << k);
                }
              if (need && (n & 31u) == 31u && (aborted(P, sm) || (int64_t)(globaltimer() - t0) > P.timeout_ns)) {
                report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_WAIT_TIMEOUT,
                             op, task, 0x40000u | (uint32_t)(g0 + __ffs(need) - 1));
                return false;
              }
            }
          }
        } else if (v == ml.nf && od.aux[0] >= 0) {   // the first routed unit: wait for this iteration's router
          const OpDev& dep = P.ops[od.aux[0]];
          if (!wait_event(P, sm, &P.events[od.aux[0]], (uint32_t)dep.ntasks * itx.g, false)) {
            report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_WAIT_TIMEOUT,
                         op, task, 0x10000u | (uint32_t)od.aux[0]);
            return false;
          }
          fence_proxy_async_global();
        }
        {
          const int u = P.units[ml.off + v];
          const int s = slot0 + u / (KP * 8), pt = (u >> 3) % KP, q = u & 7, nl = unit_lanes(q, l8);
          const int e = s >= fixed0 ? (int)I_(od, MK_I_MU_EXP0) + (s - fixed0)
                        : mtag ? (int)(((s - slot0 < 8 ? rexp_lo : rexp_hi) >> (8 * ((s - slot0) & 7))) & 0xFFu)
                               : __ldcg(mask + s);
          if (e < 0 || e >= nexp) { report_error(P, sm, MK_DERR_BAD_EXPERT, op, task, (uint32_t)e); return false; }
          const uint8_t* w13 = W13 + (size_t)e * 2 * I * H * eb;
          for (int j = 0; j < nl; ++j) {
            const size_t row0 = 2 * (size_t)(pt * Lp + 8 * (q + 8 * j));
            for (int r = 0; r < 16; r += r13)
              if (!issue_stage(P, sm, pr, w13 + (row0 + r) * H * eb, (uint32_t)(r13 * H * eb), nullptr, 0, 0, op,
                               task, e))   // the stage carries its expert (the FP8 scales are per expert)
                return false;
          }
          const uint8_t* w2 =
              W2F + ((size_t)e * H * I + (size_t)pt * H * Lp + (size_t)H * unit_q_vals(q, l8)) * eb;
          const int rb = 8 * nl * (int)eb, r2 = unit_w2_rows(rb);
          for (int r = 0; r < H; r += r2)
            if (!issue_stage(P, sm, pr, w2 + (size_t)r * rb, (uint32_t)(min(r2, H - r) * rb), nullptr, 0, 0, op, task))
              return false;
        }
      }
      return true;
    }
    case MK_OP_MLA_ATTEND: {
      const AttSplit a = att_split(od, t, itx.pos);
      if (od.op.flags & MK_F_TC) {   // TMA boxes of 24 rows, in chunks of TC_CHUNK rows
        const uint8_t* tm = reinterpret_cast<const uint8_t*>(P.tmaps) + (size_t)od.aux[2] * 256;
        const int rows = a.hi - a.lo;
        for (int c0 = 0; c0 < rows; c0 += TC_CHUNK) {
          const int nt = max(0, min(TC_CHUNK, a.n_str - c0));
          for (int r = 0; r < nt; r += TC_RPS)
            if (!issue_stage_tma(P, sm, pr, tm, tm + 128, a.lo + c0 + r, op, task)) return false;
        }
        return true;
      }
      const int DC = (int)I_(od, MK_I_ATT_DC), DR = (int)I_(od, MK_I_ATT_DR);
      const int rps = att_rps(od);
      const uint8_t* ckv = P_<const uint8_t>(od, MK_P_ATT_CKV);
      const uint8_t* kpe = P_<const uint8_t>(od, MK_P_ATT_KPE);
      for (int r = 0; r < a.n_str; r += rps) {
        const int nr = min(rps, a.n_str - r);
        const int row = a.lo + r;
        if (!issue_stage(P, sm, pr, ckv + (size_t)row * DC * 2, (uint32_t)(nr * DC * 2), kpe + (size_t)row * DR * 2,
                         (uint32_t)(nr * DR * 2), (uint32_t)(rps * DC * 2), op, task))
          return false;
      }
      return true;
    }
    default:
      return true;
  }
}

__device__ void producer_main(const KernelParams& P, Smem& sm) {
  Prod pr{0u};
  const uint32_t b = P.cta_off[blockIdx.x], e = P.cta_off[blockIdx.x + 1];
  bool ok = true;
  for (int it = 0; it < P.iters && ok; ++it) {
    Iter itx{it, P.step + 1 + it, P.gen0 + (uint32_t)it};
    for (uint32_t k = b; k < e && ok; ++k) {
      const TaskDev t = P.ctask[k].t;
      ok = produce_task(P, sm, pr, P.ops[t.op], t, itx);
    }
  }
  if (!ok) {
    // drain: the copies still in flight must land before the CTA's shared memory goes away. Each
    // outstanding stage gets the full bound of its own; a stage that still has not landed is
    // counted (Status::undrained) and reported as a ring timeout with info 3 (copies may be in
    // flight) unless an error was reported first
    uint32_t undrained = 0;
    for (uint32_t i = (pr.p_it > (uint32_t)NSTAGES ? pr.p_it - NSTAGES : 0u); i < pr.p_it; ++i) {
      const uint32_t st = i % NSTAGES, ph = (i / NSTAGES) & 1u;
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&sm.full[st], ph)) {
        if ((int64_t)(globaltimer() - t0) > P.timeout_ns) { ++undrained; break; }
      }
    }
    if (undrained) {
      atomicAdd(&P.status->undrained, undrained);
      report_error(P, sm, MK_DERR_RING_TIMEOUT, 0xFFFFFFFFu, 0xFFFFFFFFu, 3u);
    }
  }
}

// =============================================================================================
// consumer operators
// =============================================================================================

// ---- embedding ------------------------------------------------------------------------------
__device__ void op_embed(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                         Cons& c) {
  const int64_t V = I_(od, MK_I_EMB_V), H = I_(od, MK_I_EMB_H);
  const int64_t* tokens = P_<const int64_t>(od, MK_P_EMB_TOKENS);
  int64_t tok = __ldcg(reinterpret_cast<const long long*>(tokens) + itx.pos);
  if (tok < 0 || tok >= V) {
    if (c.tid == 0) report_error(P, sm, MK_DERR_TOKEN_RANGE, (uint32_t)t.op, 0, (uint32_t)tok);
    tok = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(P_<const uint16_t>(od, MK_P_EMB_W) + tok * H);
  uint4* dst = reinterpret_cast<uint4*>(P_<uint16_t>(od, MK_P_EMB_OUT));
  for (int i = c.tid; i < (int)(H / 8); i += NUM_CONSUMERS) dst[i] = __ldg(src + i);
}

// ---- copy (the debug residual snapshot) -------------------------------------------------------
__device__ void op_copy(const OpDev& od, Cons& c) {
  const int64_t n = I_(od, MK_I_CP_N);
  const uint4* src = reinterpret_cast<const uint4*>(P_<const uint16_t>(od, MK_P_CP_SRC));
  uint4* dst = reinterpret_cast<uint4*>(P_<uint16_t>(od, MK_P_CP_DST));
  for (int64_t i = c.tid; i < n / 8; i += NUM_CONSUMERS) dst[i] = ldcg16(src + i);
}

// ---- the row-dot engine ---------------------------------------------------------------------
// A row of K <= 2048 values is KS equal parts of Lp = K / KS <= 256 values (KS the fewest of 1, 2,
// 4, 8 that fit); lane l holds the 8-value vector l of a part (lanes l >= Lp / 8 hold none), adds
// the even products into a0 and the odd ones into a1, then a0 + a1, and the butterfly sums the
// lanes. In a stage of nr rows, warp w takes part p = w % KS of rows w / KS, w / KS + 8 / KS, ...
// in batches of eight that one warp_butterfly8 reduces together; the part sums go to
// pbuf[local_row * KS + p] and row_total() adds a row's parts in order (oracle detmath.dot_rows).
__device__ __forceinline__ int parts_of(int K) { return K <= 256 ? 1 : K <= 512 ? 2 : K <= 1024 ? 4 : 8; }

// this warp's x vector: part w % KS, vector `lane` (zero where the part has none)
// KS 0: the part count is a run-time value (parts_of(K)); one compact instantiation serves every
// K that the unrolled 8-part path (K of 1,025..2,048, the model's K) does not.
template <int KS>
__device__ __forceinline__ int ks_of(int K) { return KS ? KS : parts_of(K); }
template <int KS, bool SMEM>
__device__ __forceinline__ uint4 x_part(const uint16_t* x, int K, const Cons& c) {
  const int ks = ks_of<KS>(K);
  const int Lp = K / ks, off = (c.warp % ks) * Lp + c.lane * 8;
  if (c.lane * 8 >= Lp) return make_uint4(0u, 0u, 0u, 0u);
  return SMEM ? lds128(smem_u32(x + off)) : ldcg16(x + off);
}

// xf(r) gives the x vector for stage row r (the warp's own part). The eight rows' loads are issued
// before any product (rows past nr and lanes past the part read in-bounds shared memory of the
// ring and are discarded), so the batch costs one shared-memory latency.
template <int KS, class XF>
__device__ __forceinline__ void stage_parts(const uint8_t* stg, int nr, int K, int row_base, float* pbuf,
                                            const Cons& c, XF&& xf) {
  const int ks = ks_of<KS>(K);
  const int RSTEP = NUM_CONSUMER_WARPS / ks;
  const int Lp = K / ks, p = c.warp % ks;
  const bool on = c.lane * 8 < Lp;
  const uint32_t s0 = smem_u32(stg) + (uint32_t)(p * Lp + c.lane * 8) * 2u;
  const uint32_t rb = (uint32_t)K * 2u;
  for (int r0 = c.warp / ks; r0 < nr; r0 += 8 * RSTEP) {
    uint4 w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = lds128(s0 + (uint32_t)(r0 + RSTEP * i) * rb);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 x = xf(r0 + RSTEP * i);
      float a0 = 0.0f, a1 = 0.0f;
      fma_bf16x2(a0, a1, w[i].x, x.x);
      fma_bf16x2(a0, a1, w[i].y, x.y);
      fma_bf16x2(a0, a1, w[i].z, x.z);
      fma_bf16x2(a0, a1, w[i].w, x.w);
      acc[i] = (on && r0 + RSTEP * i < nr) ? __fadd_rn(a0, a1) : 0.0f;
    }
    const float d = warp_butterfly8(acc, c.lane);
    const int r = r0 + RSTEP * butterfly8_value(c.lane);
    if ((c.lane & 3) == 0 && r < nr) pbuf[(size_t)(row_base + r) * ks + p] = d;
  }
}
// stage_parts for rows of E4M3 weights (one byte each) against FP16 activations x16: the same
// lanes, parts, batches and butterfly, each lane's eight products through lane_fp8.
template <int KS>
__device__ __forceinline__ void stage_parts_fp8(const uint8_t* stg, int nr, int K, int row_base, float* pbuf,
                                                const Cons& c, uint4 x16) {
  const int ks = ks_of<KS>(K);
  const int RSTEP = NUM_CONSUMER_WARPS / ks;
  const int Lp = K / ks, p = c.warp % ks;
  const bool on = c.lane * 8 < Lp;
  const uint32_t s0 = smem_u32(stg) + (uint32_t)(p * Lp + c.lane * 8);
  const uint32_t rb = (uint32_t)K;
  for (int r0 = c.warp / ks; r0 < nr; r0 += 8 * RSTEP) {
    uint2 w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = lds64(s0 + (uint32_t)(r0 + RSTEP * i) * rb);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float v = lane_fp8(w[i], x16);
      acc[i] = (on && r0 + RSTEP * i < nr) ? v : 0.0f;
    }
    const float d = warp_butterfly8(acc, c.lane);
    const int r = r0 + RSTEP * butterfly8_value(c.lane);
    if ((c.lane & 3) == 0 && r < nr) pbuf[(size_t)(row_base + r) * ks + p] = d;
  }
}
__device__ __forceinline__ uint4 bf16x8_to_f16x8(uint4 v) {
  return make_uint4(bf16x2_to_f16x2(v.x), bf16x2_to_f16x2(v.y), bf16x2_to_f16x2(v.z), bf16x2_to_f16x2(v.w));
}
template <int KS>
__device__ __forceinline__ float row_total(const float* pbuf, int lr, int ks) {
  if constexpr (KS > 0) {
    float d = pbuf[(size_t)lr * KS];
#pragma unroll
    for (int p = 1; p < KS; ++p) d = __fadd_rn(d, pbuf[(size_t)lr * KS + p]);
    return d;
  } else {
    float d = pbuf[(size_t)lr * ks];
    for (int p = 1; p < ks; ++p) d = __fadd_rn(d, pbuf[(size_t)lr * ks + p]);
    return d;
  }
}
__device__ __forceinline__ float* pbuf_of(Smem& sm) { return reinterpret_cast<float*>(sm.scratch + PBUF_OFF); }
__device__ __forceinline__ uint16_t* xbuf_of(Smem& sm) { return reinterpret_cast<uint16_t*>(sm.scratch); }

// ---- GEMV (norm prologue, residual, fused argmax) --------------------------------------------
template <int KS>
__device__ void gemv_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                          Cons& c) {
  const int K = (int)I_(od, MK_I_GEMV_K);
  const int flags = od.op.flags;
  const uint16_t* x = P_<const uint16_t>(od, MK_P_GEMV_X);
  float* pbuf = pbuf_of(sm);
  uint4 xv;
  if (flags & MK_F_NORM) {
    uint16_t* hbuf = xbuf_of(sm);
    rmsnorm_to_smem(x, P_<const uint16_t>(od, MK_P_GEMV_WNORM), K, (float)od.op.fp[0], hbuf, sm, c);
    uint16_t* hout = P_<uint16_t>(od, MK_P_GEMV_HOUT);
    if (hout && t.idx == 0)
      for (int i = c.tid; i < K; i += NUM_CONSUMERS) hout[i] = hbuf[i];
    xv = x_part<KS, true>(hbuf, K, c);
  } else {
    xv = x_part<KS, false>(x, K, c);
  }
  // the residual of each thread's first row is read before the stages, off the epilogue's path
  const uint16_t* res = P_<const uint16_t>(od, MK_P_GEMV_RES);
  const bool has_res = (flags & MK_F_RESIDUAL) != 0;
  const float res0 = (has_res && c.tid < t.b - t.a) ? bf16_bits_to_f32(ldcg_u16(res + t.a + c.tid)) : 0.0f;
  mark_body(sm, c);
  for (int r0 = t.a; r0 < t.b; r0 += od.rps) {
    const int nr = min(od.rps, t.b - r0);
    const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    stage_parts<KS>(stg, nr, K, r0 - t.a, pbuf, c, [&](int) { return xv; });
    release_stage(sm, c);
  }
  mark_stages(sm, c);
  consumer_sync();
  uint16_t* out = P_<uint16_t>(od, MK_P_GEMV_OUT);
  const bool argmax = (flags & MK_F_ARGMAX) != 0;
  float best_v = -__int_as_float(0x7F800000);
  int best_i = 0x7FFFFFFF;
  for (int lr = c.tid; lr < t.b - t.a; lr += NUM_CONSUMERS) {
    const int row = t.a + lr;
    float d = row_total<KS>(pbuf, lr, ks_of<KS>(K));
    if (has_res) d = __fadd_rn(d, lr == c.tid ? res0 : bf16_bits_to_f32(ldcg_u16(res + row)));
    const uint32_t bits = f32_to_bf16_bits(d);
    out[row] = (uint16_t)bits;
    if (argmax) {
      const float v = bf16_bits_to_f32(bits);
      if (v > best_v || (v == best_v && row < best_i)) { best_v = v; best_i = row; }
    }
  }
  if (!argmax) return;
  // task best (ties to the lower index) -> partial slot; the last task to arrive picks the token
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
  }
  if (c.lane == 0) { sm.wbest_v[c.warp] = best_v; sm.wbest_i[c.warp] = best_i; }
  consumer_sync();
  if (c.tid == 0) {
    float v = sm.wbest_v[0];
    int i = sm.wbest_i[0];
    for (int k = 1; k < NUM_CONSUMER_WARPS; ++k)
      if (sm.wbest_v[k] > v || (sm.wbest_v[k] == v && sm.wbest_i[k] < i)) { v = sm.wbest_v[k]; i = sm.wbest_i[k]; }
    P.amax_val[t.idx] = v;
    P.amax_idx[t.idx] = i;
    // acq_rel: releases the partials above (and, through the barrier, the CTA's rows), acquires
    // every earlier task's
    const uint32_t old = atom_add_acqrel(&P.arrive[t.op], 1u);
    sm.bcast[1] = (old + 1u == (uint32_t)od.ntasks * itx.g) ? 1 : 0;
  }
  consumer_sync();
  if (!sm.bcast[1] || c.warp != 0) return;
  // the last task to arrive: warp 0 reduces all tasks' bests (lanes load in parallel; the
  // maximum with ties to the lower index does not depend on the order). Thread 0's acquire and
  // the barrier order the loads after every task's release.
  float v = -__int_as_float(0x7F800000);
  int i = 0x7FFFFFFF;
  for (int k = c.lane; k < od.ntasks; k += 32) {
    const float vk = __ldcg(P.amax_val + k);
    const int ik = __ldcg(P.amax_idx + k);
    if (vk > v || (vk == v && ik < i)) { v = vk; i = ik; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  if (c.lane == 0) {
    int64_t* tokens = P_<int64_t>(od, MK_P_GEMV_TOKENS);
    tokens[itx.pos + 1] = (int64_t)i;
    if (P.meta_step && itx.it == P.iters - 1) *P.meta_step = P.step + P.iters;
  }
}

// K > 2048 (layer 0's down projection, K = I_DENSE): one row per stage, the eight warps each
// take K / 8 of it, and the eight FP32 parts meet in shared memory (added in part order).
template <int MAXV>
__device__ void gemv_wide_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                               Cons& c) {
  const int K = (int)I_(od, MK_I_GEMV_K);
  const int flags = od.op.flags;
  const int kpart = K / NUM_CONSUMER_WARPS;
  uint4 xr[MAXV];
  load_x<MAXV, false>(xr, P_<const uint16_t>(od, MK_P_GEMV_X) + (size_t)c.warp * kpart, kpart, c.lane);
  float* pbuf = pbuf_of(sm);
  (void)itx;
  for (int r0 = t.a; r0 < t.b; ++r0) {
    const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    const float d = row_dot<MAXV>(xr, stg + (size_t)c.warp * kpart * 2, kpart, c.lane);
    if (c.lane == 0) pbuf[(size_t)(r0 - t.a) * NUM_CONSUMER_WARPS + c.warp] = d;
    release_stage(sm, c);
  }
  consumer_sync();
  const uint16_t* res = P_<const uint16_t>(od, MK_P_GEMV_RES);
  uint16_t* out = P_<uint16_t>(od, MK_P_GEMV_OUT);
  for (int lr = c.tid; lr < t.b - t.a; lr += NUM_CONSUMERS) {
    float d = row_total<NUM_CONSUMER_WARPS>(pbuf, lr, NUM_CONSUMER_WARPS);
    if (flags & MK_F_RESIDUAL) d = __fadd_rn(d, bf16_bits_to_f32(ldcg_u16(res + t.a + lr)));
    out[t.a + lr] = (uint16_t)f32_to_bf16_bits(d);
  }
}

// ---- MLA prep: cache append, RoPE, ql_nope = q_nope W_uk -------------------------------------
__device__ void op_prep(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                        Cons& c) {
  const int NH = (int)I_(od, MK_I_PREP_NH), DN = (int)I_(od, MK_I_PREP_DN), DR = (int)I_(od, MK_I_PREP_DR),
            DC = (int)I_(od, MK_I_PREP_DC);
  const int qd = DN + DR, q_out = NH * qd;
  const uint16_t* qkva = P_<const uint16_t>(od, MK_P_PREP_QKVA);
  const uint16_t* cosr = P_<const uint16_t>(od, MK_P_PREP_COS) + (size_t)itx.pos * DR;
  const uint16_t* sinr = P_<const uint16_t>(od, MK_P_PREP_SIN) + (size_t)itx.pos * DR;
  if (t.idx == 0) {
    uint16_t* hbuf = xbuf_of(sm);
    rmsnorm_to_smem(qkva + q_out, P_<const uint16_t>(od, MK_P_PREP_WKVNORM), DC, (float)od.op.fp[0], hbuf, sm, c);
    uint16_t* ckv = P_<uint16_t>(od, MK_P_PREP_CKV) + (size_t)itx.pos * DC;
    for (int i = c.tid; i < DC; i += NUM_CONSUMERS) ckv[i] = hbuf[i];
    uint16_t* kpe = P_<uint16_t>(od, MK_P_PREP_KPE) + (size_t)itx.pos * DR;
    for (int i = c.tid; i < DR; i += NUM_CONSUMERS) kpe[i] = rope_elem(qkva + q_out + DC, cosr, sinr, DR, i, true);
  }
  // q_pe of head h by tasks h, h + ntasks, ... (one head per task at the full grid)
  uint16_t* qpe = P_<uint16_t>(od, MK_P_PREP_QPE);
  for (int h = t.idx; h < NH; h += od.ntasks)
    for (int i = c.tid; i < DR; i += NUM_CONSUMERS) qpe[h * DR + i] = rope_elem(qkva + h * qd + DN, cosr, sinr, DR, i, true);
  // the W_uk product over rows [a, b) of W_ukT [NH * DC, DN]; x is the row's head's q_nope
  float* pbuf = pbuf_of(sm);
  // a task's rows touch at most two heads (tasks of at most DC rows): both heads' q_nope are
  // loaded before the stages. DN <= 256: one part per row.
  const int hf = t.a / DC, hb = (hf + 1) * DC;   // first row of the second head
  const uint4 xv0 = x_part<1, false>(qkva + hf * qd, DN, c);
  const uint4 xv1 = x_part<1, false>(qkva + min(hf + 1, NH - 1) * qd, DN, c);
  mark_body(sm, c);
  for (int r0 = t.a; r0 < t.b; r0 += od.rps) {
    const int nr = min(od.rps, t.b - r0), bnd = hb - r0;
    const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    stage_parts<1>(stg, nr, DN, r0 - t.a, pbuf, c, [&](int r) { return r < bnd ? xv0 : xv1; });
    release_stage(sm, c);
  }
  mark_stages(sm, c);
  consumer_sync();
  uint16_t* qln = P_<uint16_t>(od, MK_P_PREP_QLNOPE);
  for (int lr = c.tid; lr < t.b - t.a; lr += NUM_CONSUMERS) qln[t.a + lr] = (uint16_t)f32_to_bf16_bits(pbuf[lr]);
}

// ---- MLA attend: split-KV partials for one head (FP32 in the specified orders) --------------
// s_r = (q . k_r) * scale with lane l adding its contiguous latent columns [l LC, l LC + LC) in
// order, then its rope columns [l RP, l RP + RP), into one accumulator and the butterfly;
// m = max s; p = det_exp(s - m); l = sum p (lane l adds rows l, l + 32, ... then the butterfly);
// o_c = (sum over rows in row order of bf16(p_r) c_kv[r][c]) / l; lse = m + det_log(l).
// The split's rows sit in consecutive ring stages (rps rows each: c_kv rows, then k_pe rows);
// the position's own row (written by mla_prep this iteration) is the split's last row and is read
// from shared scratch. FAST: DC = 512 and DR = 64 (16-byte latent and 4-byte rope loads per lane).
constexpr int FAST_RPS = STAGE_BYTES / ((512 + 64) * 2);   // cache rows per stage at DC 512, DR 64
struct RowWalk {   // stage-major position of a split row, advanced without division
  uint32_t base;   // shared address of the current stage
  int slot, idx, s;
};
template <bool FAST>
__device__ void attend_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                            Cons& c) {
  const int NH = (int)I_(od, MK_I_ATT_NH), DC = (int)I_(od, MK_I_ATT_DC), DR = (int)I_(od, MK_I_ATT_DR);
  const int S = (int)I_(od, MK_I_ATT_SPLIT), prow = (int)I_(od, MK_I_ATT_PROW);
  const float scale = (float)od.op.fp[0];
  const int h = t.a, j = t.b;
  float* partials = P_<float>(od, MK_P_ATT_PARTIALS);
  float* prow_out = partials + ((size_t)j * NH + h) * prow;
  const AttSplit a = att_split(od, t, itx.pos);
  if (a.hi <= a.lo) {   // no live row at this position: o = 0, lse = -inf
    for (int i = c.tid; i < DC; i += NUM_CONSUMERS) prow_out[i] = 0.0f;
    if (c.tid == 0) prow_out[DC] = -__int_as_float(0x7F800000);
    return;
  }
  const int rows = a.hi - a.lo, nstr = a.n_str;
  const int rps = att_rps(od);
  // shared scratch: the own row, scores, bf16(p), p, m and l
  uint16_t* xrow = reinterpret_cast<uint16_t*>(sm.scratch);                 // DC + DR
  float* sc = reinterpret_cast<float*>(sm.scratch + 4096);                  // S scores
  float* pb = sc + S;                                                       // S bf16(p) as FP32
  float* pr = pb + S;                                                       // S p
  float* ml = pr + S;                                                       // m, l
  uint16_t* pbh = reinterpret_cast<uint16_t*>(ml + 4);                      // S bf16(p) as BF16 bits
  if (a.has_pos) {
    const uint16_t* ck = P_<const uint16_t>(od, MK_P_ATT_CKV) + (size_t)itx.pos * DC;
    const uint16_t* kp = P_<const uint16_t>(od, MK_P_ATT_KPE) + (size_t)itx.pos * DR;
    for (int i = c.tid; i < DC + DR; i += NUM_CONSUMERS) xrow[i] = (uint16_t)(i < DC ? ldcg_u16(ck + i) : ldcg_u16(kp + i - DC));
  }
  // q: lane l's latent columns [l LC, l LC + LC) and rope columns [l RP, l RP + RP)
  const uint16_t* qln = P_<const uint16_t>(od, MK_P_ATT_QLNOPE) + (size_t)h * DC;
  const uint16_t* qpe = P_<const uint16_t>(od, MK_P_ATT_QPE) + (size_t)h * DR;
  const int LC = DC / 32, RP = DR >= 32 ? DR / 32 : 1;
  constexpr int MC = FAST ? 1 : 4, MR = 2;
  float qn[MC], qp[MR];
  uint32_t qw[8], qpw = 0u;   // FAST: q as BF16 pairs (mixed-precision FMAs)
  if constexpr (FAST) {
    const uint4 u0 = ldcg16(qln + c.lane * 16), u1 = ldcg16(qln + c.lane * 16 + 8);
    qw[0] = u0.x; qw[1] = u0.y; qw[2] = u0.z; qw[3] = u0.w; qw[4] = u1.x; qw[5] = u1.y; qw[6] = u1.z; qw[7] = u1.w;
    qpw = __ldcg(reinterpret_cast<const unsigned int*>(qpe + c.lane * 2));
    (void)qn;
    (void)qp;
  } else {
#pragma unroll
    for (int m = 0; m < MC; ++m) qn[m] = m < LC ? bf16_bits_to_f32(ldcg_u16(qln + c.lane * LC + m)) : 0.0f;
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      const int col = c.lane * RP + m;
      qp[m] = (m < RP && col < DR) ? bf16_bits_to_f32(ldcg_u16(qpe + col)) : 0.0f;
    }
  }
  const int nst = (nstr + rps - 1) / rps;
  const uint32_t first = c.c_it;
  for (int s = 0; s < nst; ++s) acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
  consumer_sync();   // xrow visible
  mark_body(sm, c);
  const uint32_t ring0 = smem_u32(sm.ring[0]), xaddr = smem_u32(xrow);
  const uint32_t kpe_off = (uint32_t)(rps * DC * 2);
  auto walk_start = [&](int slot) {
    RowWalk w;
    w.idx = (int)(first % NSTAGES);
    w.base = ring0 + (uint32_t)w.idx * STAGE_BYTES;
    w.slot = slot;
    w.s = 0;
    return w;
  };
  auto walk_step = [&](RowWalk& w, int n) {   // n <= rps rows on
    w.slot += n;
    if (w.slot >= rps) {
      w.slot -= rps;
      ++w.s;
      w.idx = w.idx + 1 == NSTAGES ? 0 : w.idx + 1;
      w.base = ring0 + (uint32_t)w.idx * STAGE_BYTES;
    }
  };
  // scores: warp w takes rows w, w + 8, ... in batches of eight (loads first, then one
  // warp_butterfly8); rows past the split are computed on the own-row buffer and dropped
  {
    RowWalk w = walk_start(c.warp);
    for (int r0 = c.warp; r0 < rows; r0 += 8 * NUM_CONSUMER_WARPS) {
      float acc[8];
      if constexpr (FAST) {
        uint4 u0[8], u1[8];
        uint32_t kr[8];
        const int idx0 = (int)(first % NSTAGES);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = r0 + NUM_CONSUMER_WARPS * i;
          const int st = r / FAST_RPS, slot = r - st * FAST_RPS;   // constant divisor: no branch
          int idx = idx0 + st;
          idx -= idx >= NSTAGES ? NSTAGES : 0;
          const uint32_t base = ring0 + (uint32_t)idx * STAGE_BYTES;
          const bool in = r < nstr;
          const uint32_t ca = (in ? base + (uint32_t)slot * 1024u : xaddr) + (uint32_t)c.lane * 32u;
          const uint32_t ka = (in ? base + (uint32_t)(FAST_RPS * 1024) + (uint32_t)slot * 128u : xaddr + 1024u) +
                              (uint32_t)c.lane * 4u;
          u0[i] = lds128(ca);
          u1[i] = lds128(ca + 16u);
          kr[i] = lds32(ka);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t uu[8] = {u0[i].x, u0[i].y, u0[i].z, u0[i].w, u1[i].x, u1[i].y, u1[i].z, u1[i].w};
          float a0 = 0.0f;
#pragma unroll
          for (int q = 0; q < 8; ++q) a0 = fma_bf16x2_seq(a0, uu[q], qw[q]);
          acc[i] = fma_bf16x2_seq(a0, kr[i], qpw);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = r0 + NUM_CONSUMER_WARPS * i;
          const bool st = r < nstr;
          const uint32_t ca = st ? w.base + (uint32_t)w.slot * (uint32_t)(DC * 2) : xaddr;
          const uint32_t ka = st ? w.base + kpe_off + (uint32_t)w.slot * (uint32_t)(DR * 2) : xaddr + (uint32_t)DC * 2u;
          const uint16_t* crow = reinterpret_cast<const uint16_t*>(__cvta_shared_to_generic(ca));
          const uint16_t* krow = reinterpret_cast<const uint16_t*>(__cvta_shared_to_generic(ka));
          float a0 = 0.0f;
#pragma unroll
          for (int m = 0; m < MC; ++m)
            if (m < LC) a0 = fmaf(bf16_bits_to_f32((uint32_t)crow[c.lane * LC + m]), qn[m], a0);
#pragma unroll
          for (int m = 0; m < MR; ++m)
            if (m < RP && c.lane * RP + m < DR) a0 = fmaf(bf16_bits_to_f32((uint32_t)krow[c.lane * RP + m]), qp[m], a0);
          acc[i] = a0;
          walk_step(w, NUM_CONSUMER_WARPS);
        }
      }
      const float d = warp_butterfly8(acc, c.lane);
      const int rl = r0 + NUM_CONSUMER_WARPS * butterfly8_value(c.lane);
      if ((c.lane & 3) == 0 && rl < rows) sc[rl] = __fmul_rn(d, scale);
    }
  }
  consumer_sync();
  if (float* dbg = P_<float>(od, MK_P_ATT_SCORES))   // debug: the scaled scores of this head's rows
    for (int r = c.tid; r < rows; r += NUM_CONSUMERS) dbg[(size_t)h * I_(od, MK_I_ATT_SMAX) + a.lo + r] = sc[r];
  // softmax: every warp finds m; thread r computes p_r; warp 0 adds l in the lane order
  float mx = -__int_as_float(0x7F800000);
  for (int r = c.lane; r < rows; r += 32) mx = fmaxf(mx, sc[r]);
  mx = warp_max_f32(mx);
  for (int r = c.tid; r < rows; r += NUM_CONSUMERS) {
    const float p = det_exp(__fsub_rn(sc[r], mx));
    pr[r] = p;
    pb[r] = round_bf16(p);
    pbh[r] = (uint16_t)(__float_as_uint(pb[r]) >> 16);
  }
  consumer_sync();
  if (c.warp == 0) {
    float sum = 0.0f;
    for (int r = c.lane; r < rows; r += 32) sum = __fadd_rn(sum, pr[r]);
    sum = warp_butterfly(sum);
    if (c.lane == 0) { ml[0] = mx; ml[1] = sum; }
  }
  // o: each thread owns pairs of adjacent latent columns and walks the rows in order
  const uint32_t pbaddr = smem_u32(pb), pbhaddr = smem_u32(pbh);
  float acc00 = 0.0f, acc01 = 0.0f, acc10 = 0.0f, acc11 = 0.0f;   // pairs k = 0, 1 (registers, not an array)
  int np = 0;
  for (int i = c.tid, k = 0; i < DC / 2 && k < 2; i += NUM_CONSUMERS, ++k) {
    const uint32_t col = (uint32_t)i * 4u;   // byte offset of the pair in a row
    float s0 = 0.0f, s1 = 0.0f;
    RowWalk w = walk_start(0);
    int r = 0;
    if constexpr (FAST) {   // stage by stage: rows at a constant stride, eight loads in flight
      int idx = (int)(first % NSTAGES);
      for (int st = 0; st < nst; ++st) {
        const uint32_t base = ring0 + (uint32_t)idx * STAGE_BYTES + col;
        idx = idx + 1 == NSTAGES ? 0 : idx + 1;
        const int n = min(FAST_RPS, nstr - r);
        int slot = 0;
        for (; slot + 8 <= n; slot += 8, r += 8) {   // r is a multiple of 4: 8-byte p loads
          uint32_t v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = lds32(base + (uint32_t)(slot + u) * 1024u);
          const uint2 pa = lds64(pbhaddr + (uint32_t)r * 2u), pc = lds64(pbhaddr + (uint32_t)r * 2u + 8u);
          fma_pv2(s0, s1, v[0], v[1], pa.x);
          fma_pv2(s0, s1, v[2], v[3], pa.y);
          fma_pv2(s0, s1, v[4], v[5], pc.x);
          fma_pv2(s0, s1, v[6], v[7], pc.y);
        }
        for (; slot < n; ++slot, ++r) fma_pv1(s0, s1, lds32(base + (uint32_t)slot * 1024u), lds16(pbhaddr + (uint32_t)r * 2u));
      }
    }
    if constexpr (!FAST) {
    for (; r + 4 <= nstr; r += 4) {          // four rows' loads in flight, then in order
      uint32_t v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        v[u] = lds32(w.base + (uint32_t)w.slot * (uint32_t)(DC * 2) + col);
        walk_step(w, 1);
      }
      const uint4 p4 = lds128(pbaddr + (uint32_t)r * 4u);
      const float pp[4] = {__uint_as_float(p4.x), __uint_as_float(p4.y), __uint_as_float(p4.z), __uint_as_float(p4.w)};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        s0 = fmaf(lo_f32(v[u]), pp[u], s0);
        s1 = fmaf(hi_f32(v[u]), pp[u], s1);
      }
    }
    for (; r < nstr; ++r) {
      const uint32_t v = lds32(w.base + (uint32_t)w.slot * (uint32_t)(DC * 2) + col);
      walk_step(w, 1);
      const float pp = ldsf(pbaddr + (uint32_t)r * 4u);
      s0 = fmaf(lo_f32(v), pp, s0);
      s1 = fmaf(hi_f32(v), pp, s1);
    }
    }   // FAST: the stage loop above covered every streamed row
    if (a.has_pos) {
      const uint32_t v = lds32(xaddr + col);
      const float pp = ldsf(pbaddr + (uint32_t)nstr * 4u);
      s0 = fmaf(lo_f32(v), pp, s0);
      s1 = fmaf(hi_f32(v), pp, s1);
    }
    if (k == 0) { acc00 = s0; acc01 = s1; } else { acc10 = s0; acc11 = s1; }
    np = k + 1;
  }
  consumer_sync();   // l
  const float l = ml[1];
  for (int k = 0; k < np; ++k) {
    const int i = c.tid + k * NUM_CONSUMERS;
    *reinterpret_cast<float2*>(prow_out + 2 * i) =
        make_float2(__fdiv_rn(k == 0 ? acc00 : acc10, l), __fdiv_rn(k == 0 ? acc01 : acc11, l));
  }
  if (c.tid == 0) prow_out[DC] = __fadd_rn(ml[0], det_log(l));
  for (int s = 0; s < nst; ++s) release_stage(sm, c);
  mark_stages(sm, c);
}

// Two heads at a time (DC 512, DR 64, an even head group): every cache row loaded from the ring
// serves both heads' scores and both heads' P.V, so a head costs half the shared-memory reads and
// each thread keeps twice the independent FMA chains in flight. Per head, every sum is the
// single-head path's, in the same order (attend_body<true>): the outputs are identical.
struct AttHead {   // one head's shared scratch: scores, bf16(p) as FP32, p, m and l, bf16(p) bits
  float *sc, *pb, *pr, *ml;
  uint16_t* pbh;
};
__device__ __forceinline__ AttHead att_head(Smem& sm, int S, int k) {
  const int blk = ((3 * S + 4) * 4 + S * 2 + 15) / 16 * 16;
  AttHead a;
  a.sc = reinterpret_cast<float*>(sm.scratch + 4096 + k * blk);
  a.pb = a.sc + S;
  a.pr = a.pb + S;
  a.ml = a.pr + S;
  a.pbh = reinterpret_cast<uint16_t*>(a.ml + 4);
  return a;
}
__device__ __forceinline__ void attend_pairs(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                             Cons& c) {
  constexpr int DC = 512, DR = 64;
  const int NH = (int)I_(od, MK_I_ATT_NH), S = (int)I_(od, MK_I_ATT_SPLIT), prow = (int)I_(od, MK_I_ATT_PROW);
  const float scale = (float)od.op.fp[0];
  const int HG = (int)I_(od, MK_I_ATT_HGROUP), j = t.b;
  float* partials = P_<float>(od, MK_P_ATT_PARTIALS);
  const AttSplit a = att_split(od, t, itx.pos);
  if (a.hi <= a.lo) {   // no live row at this position: o = 0, lse = -inf
    for (int hh = 0; hh < HG; ++hh) {
      float* prow_out = partials + ((size_t)j * NH + t.a * HG + hh) * prow;
      for (int i = c.tid; i < DC; i += NUM_CONSUMERS) prow_out[i] = 0.0f;
      if (c.tid == 0) prow_out[DC] = -__int_as_float(0x7F800000);
    }
    return;
  }
  const int rows = a.hi - a.lo, nstr = a.n_str;
  uint16_t* xrow = reinterpret_cast<uint16_t*>(sm.scratch);   // the own row: DC + DR
  const AttHead H0 = att_head(sm, S, 0), H1 = att_head(sm, S, 1);
  if (a.has_pos) {
    const uint16_t* ck = P_<const uint16_t>(od, MK_P_ATT_CKV) + (size_t)itx.pos * DC;
    const uint16_t* kp = P_<const uint16_t>(od, MK_P_ATT_KPE) + (size_t)itx.pos * DR;
    for (int i = c.tid; i < DC + DR; i += NUM_CONSUMERS) xrow[i] = (uint16_t)(i < DC ? ldcg_u16(ck + i) : ldcg_u16(kp + i - DC));
  }
  const int nst = (nstr + FAST_RPS - 1) / FAST_RPS;
  const uint32_t first = c.c_it;
  const uint32_t ring0 = smem_u32(sm.ring[0]), xaddr = smem_u32(xrow);
  const int idx0 = (int)(first % NSTAGES);
  for (int hp = 0; hp < HG; hp += 2) {
    const int hA = t.a * HG + hp, hB = hA + 1;
    // q of both heads as BF16 pairs: lane l's latent columns [16 l, 16 l + 16), rope columns 2 l, 2 l + 1
    uint32_t qa[8], qb[8];
    {
      const uint16_t* qln = P_<const uint16_t>(od, MK_P_ATT_QLNOPE);
      const uint4 a0 = ldcg16(qln + (size_t)hA * DC + c.lane * 16), a1 = ldcg16(qln + (size_t)hA * DC + c.lane * 16 + 8);
      const uint4 b0 = ldcg16(qln + (size_t)hB * DC + c.lane * 16), b1 = ldcg16(qln + (size_t)hB * DC + c.lane * 16 + 8);
      qa[0] = a0.x; qa[1] = a0.y; qa[2] = a0.z; qa[3] = a0.w; qa[4] = a1.x; qa[5] = a1.y; qa[6] = a1.z; qa[7] = a1.w;
      qb[0] = b0.x; qb[1] = b0.y; qb[2] = b0.z; qb[3] = b0.w; qb[4] = b1.x; qb[5] = b1.y; qb[6] = b1.z; qb[7] = b1.w;
    }
    const uint16_t* qpe = P_<const uint16_t>(od, MK_P_ATT_QPE);
    const uint32_t qpa = __ldcg(reinterpret_cast<const unsigned int*>(qpe + (size_t)hA * DR + c.lane * 2));
    const uint32_t qpb = __ldcg(reinterpret_cast<const unsigned int*>(qpe + (size_t)hB * DR + c.lane * 2));
    if (hp == 0) {
      for (int st = 0; st < nst; ++st) acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
      consumer_sync();   // xrow visible
      mark_body(sm, c);
    }
    // scores: warp w takes rows w, w + 8, ... in batches of eight; one row load, two heads
    for (int r0 = c.warp; r0 < rows; r0 += 8 * NUM_CONSUMER_WARPS) {
      uint4 u0[8], u1[8];
      uint32_t kr[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = r0 + NUM_CONSUMER_WARPS * i;
        const int st = r / FAST_RPS, slot = r - st * FAST_RPS;
        int idx = idx0 + st;
        idx -= idx >= NSTAGES ? NSTAGES : 0;
        const uint32_t base = ring0 + (uint32_t)idx * STAGE_BYTES;
        const bool in = r < nstr;
        const uint32_t ca = (in ? base + (uint32_t)slot * 1024u : xaddr) + (uint32_t)c.lane * 32u;
        const uint32_t ka = (in ? base + (uint32_t)(FAST_RPS * 1024) + (uint32_t)slot * 128u : xaddr + 1024u) +
                            (uint32_t)c.lane * 4u;
        u0[i] = lds128(ca);
        u1[i] = lds128(ca + 16u);
        kr[i] = lds32(ka);
      }
      float acca[8], accb[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t uu[8] = {u0[i].x, u0[i].y, u0[i].z, u0[i].w, u1[i].x, u1[i].y, u1[i].z, u1[i].w};
        float x0 = 0.0f, y0 = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          x0 = fma_bf16x2_seq(x0, uu[q], qa[q]);
          y0 = fma_bf16x2_seq(y0, uu[q], qb[q]);
        }
        acca[i] = fma_bf16x2_seq(x0, kr[i], qpa);
        accb[i] = fma_bf16x2_seq(y0, kr[i], qpb);
      }
      const float da = warp_butterfly8(acca, c.lane);
      const float db = warp_butterfly8(accb, c.lane);
      const int rl = r0 + NUM_CONSUMER_WARPS * butterfly8_value(c.lane);
      if ((c.lane & 3) == 0 && rl < rows) {
        H0.sc[rl] = __fmul_rn(da, scale);
        H1.sc[rl] = __fmul_rn(db, scale);
      }
    }
    consumer_sync();
    if (float* dbg = P_<float>(od, MK_P_ATT_SCORES))   // debug: the scaled scores of both heads' rows
      for (int u = c.tid; u < 2 * rows; u += NUM_CONSUMERS)
        dbg[(size_t)(u < rows ? hA : hB) * I_(od, MK_I_ATT_SMAX) + a.lo + (u < rows ? u : u - rows)] =
            u < rows ? H0.sc[u] : H1.sc[u - rows];
    // softmax: every warp finds both maxima; thread u computes p of row u mod rows of head u / rows
    float ma = -__int_as_float(0x7F800000), mb = ma;
    for (int r = c.lane; r < rows; r += 32) {
      ma = fmaxf(ma, H0.sc[r]);
      mb = fmaxf(mb, H1.sc[r]);
    }
    ma = warp_max_f32(ma);
    mb = warp_max_f32(mb);
    for (int u = c.tid; u < 2 * rows; u += NUM_CONSUMERS) {
      const bool second = u >= rows;
      const AttHead& Hd = second ? H1 : H0;
      const int r = second ? u - rows : u;
      const float p = det_exp(__fsub_rn(Hd.sc[r], second ? mb : ma));
      Hd.pr[r] = p;
      Hd.pb[r] = round_bf16(p);
      Hd.pbh[r] = (uint16_t)(__float_as_uint(Hd.pb[r]) >> 16);
    }
    consumer_sync();
    if (c.warp < 2) {   // warp 0 adds head A's l, warp 1 head B's, each in the lane order
      const AttHead& Hd = c.warp ? H1 : H0;
      float sum = 0.0f;
      for (int r = c.lane; r < rows; r += 32) sum = __fadd_rn(sum, Hd.pr[r]);
      sum = warp_butterfly(sum);
      if (c.lane == 0) { Hd.ml[0] = c.warp ? mb : ma; Hd.ml[1] = sum; }
    }
    // o: thread t owns latent column pair t of both heads and walks the rows in order
    const uint32_t col = (uint32_t)c.tid * 4u;
    const uint32_t pha = smem_u32(H0.pbh), phb = smem_u32(H1.pbh);
    float s0 = 0.0f, s1 = 0.0f, t0 = 0.0f, t1 = 0.0f;
    {
      int r = 0, idx = idx0;
      for (int st = 0; st < nst; ++st) {
        const uint32_t base = ring0 + (uint32_t)idx * STAGE_BYTES + col;
        idx = idx + 1 == NSTAGES ? 0 : idx + 1;
        const int n = min(FAST_RPS, nstr - r);
        int slot = 0;
        for (; slot + 8 <= n; slot += 8, r += 8) {   // r is a multiple of 4: 8-byte p loads
          uint32_t v[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) v[u] = lds32(base + (uint32_t)(slot + u) * 1024u);
          const uint2 pa = lds64(pha + (uint32_t)r * 2u), pc = lds64(pha + (uint32_t)r * 2u + 8u);
          const uint2 qa2 = lds64(phb + (uint32_t)r * 2u), qc2 = lds64(phb + (uint32_t)r * 2u + 8u);
          fma_pv2(s0, s1, v[0], v[1], pa.x);
          fma_pv2(t0, t1, v[0], v[1], qa2.x);
          fma_pv2(s0, s1, v[2], v[3], pa.y);
          fma_pv2(t0, t1, v[2], v[3], qa2.y);
          fma_pv2(s0, s1, v[4], v[5], pc.x);
          fma_pv2(t0, t1, v[4], v[5], qc2.x);
          fma_pv2(s0, s1, v[6], v[7], pc.y);
          fma_pv2(t0, t1, v[6], v[7], qc2.y);
        }
        for (; slot < n; ++slot, ++r) {
          const uint32_t v = lds32(base + (uint32_t)slot * 1024u);
          fma_pv1(s0, s1, v, lds16(pha + (uint32_t)r * 2u));
          fma_pv1(t0, t1, v, lds16(phb + (uint32_t)r * 2u));
        }
      }
    }
    if (a.has_pos) {
      const uint32_t v = lds32(xaddr + col);
      const float pa = H0.pb[nstr], pb = H1.pb[nstr];
      s0 = fmaf(lo_f32(v), pa, s0);
      s1 = fmaf(hi_f32(v), pa, s1);
      t0 = fmaf(lo_f32(v), pb, t0);
      t1 = fmaf(hi_f32(v), pb, t1);
    }
    consumer_sync();   // l of both heads
    {
      const float la = H0.ml[1], lb = H1.ml[1];
      float* oa = partials + ((size_t)j * NH + hA) * prow;
      float* ob = partials + ((size_t)j * NH + hB) * prow;
      *reinterpret_cast<float2*>(oa + 2 * c.tid) = make_float2(__fdiv_rn(s0, la), __fdiv_rn(s1, la));
      *reinterpret_cast<float2*>(ob + 2 * c.tid) = make_float2(__fdiv_rn(t0, lb), __fdiv_rn(t1, lb));
      if (c.tid == 0) oa[DC] = __fadd_rn(H0.ml[0], det_log(la));
      if (c.tid == 32) ob[DC] = __fadd_rn(H1.ml[0], det_log(lb));
    }
    // the next pair may overwrite the scores and p at once: every thread has passed the barrier
    // after P.V, and m and l are rewritten only after the next pair's second barrier
  }
  for (int st = 0; st < nst; ++st) release_stage(sm, c);
  mark_stages(sm, c);
}

// ---- MLA attend on the tensor cores (MK_F_TC): all heads of one split per task ---------------
// The split's cache rows stream through the ring as TMA boxes with the 128-byte swizzle (a stage:
// 24 rows x 8 latent boxes of 64 columns + 1 rope box), in chunks of up to four stages (96 rows).
// Per chunk: S = Q K^T for the 16 heads (mma.m16n8k16: heads are M, cache rows N, the 576 latent
// + rope columns K; Q from shared memory, K straight from the swizzled stages by ldmatrix), an
// online softmax across chunks (running max and sum per head, det_exp), P rounded to BF16 (the
// reference's rounding point) and O += P V (rows are K, latent columns N, V = the same stages read
// with ldmatrix.trans). The last chunk's own row (written by mla_prep this iteration) and rows
// past the split are read from an own-row buffer and a zero chunk instead of the ring. FP32
// accumulation in the tensor cores' order, so the partials agree with the specified-order path
// within rounding, not bit for bit.
struct TcRow {      // one row of a chunk: the shared address of its column c is
  uint32_t base;     //   base + (c >> 6) * box + ((((c & 63) >> 3) ^ key) << 4 & mask)
  uint32_t box, key, mask;
  __device__ __forceinline__ uint32_t at(int c) const {
    return base + (uint32_t)(c >> 6) * box + (((((uint32_t)c & 63u) >> 3) ^ key) << 4 & mask);
  }
};
struct TcRows {    // where a chunk's rows are: nt streamed rows in ring stages from index idx0
  uint32_t ring0, own, zero;
  int idx0, nt, own_r;
  __device__ __forceinline__ TcRow row(int r) const {
    TcRow w;
    if (r < nt) {              // a swizzled stage row: 64-column boxes of TC_BOX bytes
      const int st = r / TC_RPS, slot = r - st * TC_RPS;
      int idx = idx0 + st;
      idx -= idx >= NSTAGES ? NSTAGES : 0;
      w.base = ring0 + (uint32_t)idx * STAGE_BYTES + (uint32_t)slot * 128u;
      w.box = TC_BOX;
      w.key = (uint32_t)(slot & 7);
      w.mask = 0xFFFFFFFFu;
    } else if (r == own_r) {   // the own row, unswizzled: 128 bytes per 64 columns
      w.base = own;
      w.box = 128u;
      w.key = 0u;
      w.mask = 0xFFFFFFFFu;
    } else {                   // past the chunk: one zero chunk
      w.base = zero;
      w.box = 0u;
      w.key = 0u;
      w.mask = 0u;
    }
    return w;
  }
};

// Out of line: its own register allocation, so the inlined operators keep theirs. The lane
// indices are copied into registers at entry (through the caller's reference they would be
// reloaded from local memory, whose lines miss the small L1 beside the shared-memory carveout).
__device__ __forceinline__ void attend_tc(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t,
                                      const Iter itx, Cons& c) {
  const int warp = c.warp, lane = c.lane, tid = c.tid;
  constexpr int DC = 512, DR = 64, NH = 16;
  const int prow = (int)I_(od, MK_I_ATT_PROW), j = t.b;
  // latent-column part q of QN: this task's P.V covers columns [q * CW, q * CW + CW)
  const int QN = (int)I_(od, MK_I_ATT_CPARTS), q = t.a, CW = DC / QN, npairs = CW / 16;
  const float scale = (float)od.op.fp[0];
  float* partials = P_<float>(od, MK_P_ATT_PARTIALS);
  const AttSplit a = att_split(od, t, itx.pos);
  const float NEG_INF = -__int_as_float(0x7F800000);
  if (a.hi <= a.lo) {   // no live row at this position: o = 0, lse = -inf
    for (int i = tid; i < NH * CW; i += NUM_CONSUMERS)
      partials[((size_t)j * NH + i / CW) * prow + q * CW + i % CW] = 0.0f;
    if (q == 0 && tid < NH) partials[((size_t)j * NH + tid) * prow + DC] = NEG_INF;
    return;
  }
  const int rows = a.hi - a.lo, nstr = a.n_str;
  uint8_t* scr = sm.scratch;
  const uint32_t qbase = smem_u32(scr + TC_Q_OFF), pbase = smem_u32(scr + TC_P_OFF);
  // Q of the 16 heads (ql_nope then q_pe), the own row and the zero chunk
  {
    const uint16_t* qln = P_<const uint16_t>(od, MK_P_ATT_QLNOPE);
    const uint16_t* qpe = P_<const uint16_t>(od, MK_P_ATT_QPE);
    for (int i = tid; i < NH * 72; i += NUM_CONSUMERS) {
      const int h = i / 72, q8 = i - h * 72;
      const uint4 v = q8 < 64 ? ldcg16(qln + (size_t)h * DC + q8 * 8) : ldcg16(qpe + (size_t)h * DR + (q8 - 64) * 8);
      *reinterpret_cast<uint4*>(scr + TC_Q_OFF + h * TC_QSTRIDE + q8 * 16) = v;
    }
    if (a.has_pos) {
      const uint16_t* ck = P_<const uint16_t>(od, MK_P_ATT_CKV) + (size_t)itx.pos * DC;
      const uint16_t* kp = P_<const uint16_t>(od, MK_P_ATT_KPE) + (size_t)itx.pos * DR;
      for (int i = tid; i < 72; i += NUM_CONSUMERS)
        *reinterpret_cast<uint4*>(scr + TC_OWN_OFF + i * 16) = i < 64 ? ldcg16(ck + i * 8) : ldcg16(kp + (i - 64) * 8);
    }
    if (tid == 0) *reinterpret_cast<uint4*>(scr + TC_ZERO_OFF) = make_uint4(0u, 0u, 0u, 0u);
  }
  float* red = reinterpret_cast<float*>(scr + TC_RED_OFF);   // [2][8 warps][16 heads]
  const int g = lane >> 2, tig = lane & 3;
  // running softmax statistics of heads g and g + 8 (every thread of a group keeps the same)
  float m_g = NEG_INF, m_g8 = NEG_INF, l_g = 0.0f, l_g8 = 0.0f;
  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  const uint32_t ring0 = smem_u32(sm.ring[0]);
  bool marked = false;
  for (int c0 = 0; c0 < rows; c0 += TC_CHUNK) {
    const int R = min(TC_CHUNK, rows - c0), nt = max(0, min(TC_CHUNK, nstr - c0));
    const int ns = (nt + TC_RPS - 1) / TC_RPS;
    TcRows tr;
    tr.ring0 = ring0;
    tr.own = smem_u32(scr + TC_OWN_OFF);
    tr.zero = smem_u32(scr + TC_ZERO_OFF);
    tr.idx0 = (int)(c.c_it % NSTAGES);
    tr.nt = nt;
    tr.own_r = (a.has_pos && nstr >= c0 && nstr < c0 + R) ? nstr - c0 : -1;
    for (int s = 0; s < ns; ++s) acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    consumer_sync();   // Q, the own row and the zero chunk are visible (first chunk)
    if (!marked) { mark_body(sm, c); marked = true; }
    // ---- S = Q K^T over 16-row pairs of the chunk: with at most four pairs, two warps share a pair
    // (the first and second half of the 36 k-steps, added through shared memory), else one warp
    // per pair; each warp keeps two accumulator sets (even and odd k-steps) so two mma chains
    // overlap
    const int pairs = (R + 15) / 16;
    const bool split_k = pairs <= 4;
    const int jp = split_k ? (warp >> 1) : warp, kh = split_k ? (warp & 1) : 0;
    // k-steps in groups of four (one 64-column box each): halves of 5 and 4 groups when split
    const int g0 = split_k ? 5 * kh : 0, g1 = split_k ? (kh ? 9 : 5) : 9;
    float mx_g = NEG_INF, mx_g8 = NEG_INF;
    float acc[2][4];
    const bool in_pair = jp < pairs;
    const bool has_pair = in_pair && kh == 0;     // this warp owns the pair's finished scores
    if (in_pair) {
      float accb[2][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[0][i] = acc[1][i] = accb[0][i] = accb[1][i] = 0.0f;
      const int qh = (lane & 7) + 8 * ((lane >> 3) & 1), qk = 8 * (lane >> 4);
      const int bk = 8 * ((lane >> 3) & 1);
      const TcRow kr = tr.row(16 * jp + (lane & 7) + 8 * (lane >> 4));
      uint32_t off[4];   // the lane's column offsets within a box for the four k-steps of a group
#pragma unroll
      for (int j = 0; j < 4; ++j) off[j] = (((uint32_t)(2 * j) + (uint32_t)(bk >> 3)) ^ kr.key) << 4 & kr.mask;
      const uint32_t qa = qbase + (uint32_t)(qh * TC_QSTRIDE + qk * 2);
#pragma unroll 1
      for (int gi = g0; gi < g1; ++gi) {
        const uint32_t kb = kr.base + (uint32_t)gi * kr.box, qg = qa + (uint32_t)gi * 128u;
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          uint32_t a0, a1, a2, a3, b0, b1, b2, b3, e0, e1, e2, e3, f0, f1, f2, f3;
          ldsm_x4(qg + (uint32_t)j * 32u, a0, a1, a2, a3);
          ldsm_x4(kb + off[j], b0, b1, b2, b3);
          ldsm_x4(qg + (uint32_t)(j + 1) * 32u, e0, e1, e2, e3);
          ldsm_x4(kb + off[j + 1], f0, f1, f2, f3);
          mma_bf16_16816(acc[0], a0, a1, a2, a3, b0, b1);
          mma_bf16_16816(acc[1], a0, a1, a2, a3, b2, b3);
          mma_bf16_16816(accb[0], e0, e1, e2, e3, f0, f1);
          mma_bf16_16816(accb[1], e0, e1, e2, e3, f2, f3);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[0][i] = __fadd_rn(acc[0][i], accb[0][i]);
        acc[1][i] = __fadd_rn(acc[1][i], accb[1][i]);
      }
      if (split_k && kh == 1) {
        float* hp = reinterpret_cast<float*>(scr + TC_HALF_OFF) + (jp * 32 + lane) * 8;
        *reinterpret_cast<float4*>(hp) = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
        *reinterpret_cast<float4*>(hp + 4) = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
      }
    }
    if (split_k) consumer_sync();   // the second halves' partial scores
    if (has_pair) {
      if (split_k) {
        const float* hp = reinterpret_cast<const float*>(scr + TC_HALF_OFF) + (jp * 32 + lane) * 8;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[0][i] = __fadd_rn(acc[0][i], hp[i]);
          acc[1][i] = __fadd_rn(acc[1][i], hp[4 + i]);
        }
      }
      // scale, mask rows past the chunk, running maxima of heads g and g + 8
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = 16 * jp + 8 * h + 2 * tig + (e & 1);
          acc[h][e] = r < R ? __fmul_rn(acc[h][e], scale) : NEG_INF;
        }
        mx_g = fmaxf(mx_g, fmaxf(acc[h][0], acc[h][1]));
        mx_g8 = fmaxf(mx_g8, fmaxf(acc[h][2], acc[h][3]));
      }
      if (float* dbg = P_<float>(od, MK_P_ATT_SCORES)) {   // debug: the scaled scores of live rows
        const int64_t smax = I_(od, MK_I_ATT_SMAX);
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int r = 16 * jp + 8 * h + 2 * tig + (e & 1);
            if (r < R) dbg[(size_t)(e < 2 ? g : g + 8) * smax + a.lo + c0 + r] = acc[h][e];
          }
      }
    }
    mx_g = fmaxf(mx_g, __shfl_xor_sync(0xffffffffu, mx_g, 1));
    mx_g = fmaxf(mx_g, __shfl_xor_sync(0xffffffffu, mx_g, 2));
    mx_g8 = fmaxf(mx_g8, __shfl_xor_sync(0xffffffffu, mx_g8, 1));
    mx_g8 = fmaxf(mx_g8, __shfl_xor_sync(0xffffffffu, mx_g8, 2));
    if (tig == 0) { red[warp * 16 + g] = mx_g; red[warp * 16 + g + 8] = mx_g8; }
    consumer_sync();
    float cm_g = NEG_INF, cm_g8 = NEG_INF;
#pragma unroll
    for (int w = 0; w < NUM_CONSUMER_WARPS; ++w) {
      cm_g = fmaxf(cm_g, red[w * 16 + g]);
      cm_g8 = fmaxf(cm_g8, red[w * 16 + g + 8]);
    }
    const float mn_g = fmaxf(m_g, cm_g), mn_g8 = fmaxf(m_g8, cm_g8);
    const float al_g = det_exp(__fsub_rn(m_g, mn_g)), al_g8 = det_exp(__fsub_rn(m_g8, mn_g8));
    // p = exp(s - m), rounded to BF16 into P[head][row]; the sums use the unrounded p
    float ls_g = 0.0f, ls_g8 = 0.0f;
    if (has_pair) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float p0 = det_exp(__fsub_rn(acc[h][0], mn_g)), p1 = det_exp(__fsub_rn(acc[h][1], mn_g));
        const float p2 = det_exp(__fsub_rn(acc[h][2], mn_g8)), p3 = det_exp(__fsub_rn(acc[h][3], mn_g8));
        ls_g = __fadd_rn(ls_g, __fadd_rn(p0, p1));
        ls_g8 = __fadd_rn(ls_g8, __fadd_rn(p2, p3));
        const int col = 16 * jp + 8 * h + 2 * tig;
        *reinterpret_cast<uint32_t*>(scr + TC_P_OFF + g * TC_PSTRIDE + col * 2) =
            f32_to_bf16_bits(p0) | (f32_to_bf16_bits(p1) << 16);
        *reinterpret_cast<uint32_t*>(scr + TC_P_OFF + (g + 8) * TC_PSTRIDE + col * 2) =
            f32_to_bf16_bits(p2) | (f32_to_bf16_bits(p3) << 16);
      }
    }
    ls_g = __fadd_rn(ls_g, __shfl_xor_sync(0xffffffffu, ls_g, 1));
    ls_g = __fadd_rn(ls_g, __shfl_xor_sync(0xffffffffu, ls_g, 2));
    ls_g8 = __fadd_rn(ls_g8, __shfl_xor_sync(0xffffffffu, ls_g8, 1));
    ls_g8 = __fadd_rn(ls_g8, __shfl_xor_sync(0xffffffffu, ls_g8, 2));
    if (tig == 0) {
      red[NUM_CONSUMER_WARPS * 16 + warp * 16 + g] = has_pair ? ls_g : 0.0f;
      red[NUM_CONSUMER_WARPS * 16 + warp * 16 + g + 8] = has_pair ? ls_g8 : 0.0f;
    }
    consumer_sync();   // P and the sums are complete
    float cs_g = 0.0f, cs_g8 = 0.0f;
#pragma unroll
    for (int w = 0; w < NUM_CONSUMER_WARPS; ++w) {
      cs_g = __fadd_rn(cs_g, red[NUM_CONSUMER_WARPS * 16 + w * 16 + g]);
      cs_g8 = __fadd_rn(cs_g8, red[NUM_CONSUMER_WARPS * 16 + w * 16 + g + 8]);
    }
    l_g = __fadd_rn(__fmul_rn(l_g, al_g), cs_g);
    l_g8 = __fadd_rn(__fmul_rn(l_g8, al_g8), cs_g8);
    m_g = mn_g;
    m_g8 = mn_g8;
    // ---- O = O alpha + P V: the part's 16-column pairs w, w + 8, ... (at most four per warp)
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      o[n][0] = __fmul_rn(o[n][0], al_g);
      o[n][1] = __fmul_rn(o[n][1], al_g);
      o[n][2] = __fmul_rn(o[n][2], al_g8);
      o[n][3] = __fmul_rn(o[n][3], al_g8);
    }
    {
      const int ph = (lane & 7) + 8 * ((lane >> 3) & 1), pk = 8 * (lane >> 4);
      const int vr = (lane & 7) + 8 * ((lane >> 3) & 1), vc = q * CW + 8 * (lane >> 4);
      for (int kk = 0; kk < pairs; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(pbase + (uint32_t)(ph * TC_PSTRIDE + (16 * kk + pk) * 2), a0, a1, a2, a3);
        const TcRow vrow = tr.row(16 * kk + vr);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int pi = warp + 8 * i;
          if (pi < npairs) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vrow.at(vc + 16 * pi), b0, b1, b2, b3);
            mma_bf16_16816(o[2 * i], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(o[2 * i + 1], a0, a1, a2, a3, b2, b3);
          }
        }
      }
    }
    consumer_sync();   // every warp is done with the chunk's stages, P and the reductions
    for (int s = 0; s < ns; ++s) release_stage(sm, c);
  }
  mark_stages(sm, c);
  // o = O / l (one reciprocal per head) and lse = m + log l into the split's partial rows
  const float il_g = __fdiv_rn(1.0f, l_g), il_g8 = __fdiv_rn(1.0f, l_g8);
  float* out_g = partials + ((size_t)j * NH + g) * prow;
  float* out_g8 = partials + ((size_t)j * NH + g + 8) * prow;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int pi = warp + 8 * i;
    if (pi < npairs) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = 2 * i + h, col = q * CW + 16 * pi + 8 * h + 2 * tig;
        *reinterpret_cast<float2*>(out_g + col) = make_float2(__fmul_rn(o[n][0], il_g), __fmul_rn(o[n][1], il_g));
        *reinterpret_cast<float2*>(out_g8 + col) = make_float2(__fmul_rn(o[n][2], il_g8), __fmul_rn(o[n][3], il_g8));
      }
    }
  }
  if (q == 0 && warp == 0 && tig == 0) {
    out_g[DC] = __fadd_rn(m_g, det_log(l_g));
    out_g8[DC] = __fadd_rn(m_g8, det_log(l_g8));
  }
}

// ---- merge of the splits + attn = W_uv o ----------------------------------------------------
template <int KS>
__device__ void merge_rows(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const uint16_t* obuf,
                           int hf, int DV, int DC, Cons& c) {
  float* pbuf = pbuf_of(sm);
  // a task's rows touch at most two heads: the warp's part of both heads' o, and the first row of
  // the second head
  const int nh_t = (t.b - 1) / DV - hf + 1, hb = (hf + 1) * DV;
  const uint4 xv0 = x_part<KS, true>(obuf, DC, c);
  const uint4 xv1 = nh_t > 1 ? x_part<KS, true>(obuf + DC, DC, c) : xv0;
  for (int r0 = t.a; r0 < t.b; r0 += od.rps) {
    const int nr = min(od.rps, t.b - r0), bnd = hb - r0;
    const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    stage_parts<KS>(stg, nr, DC, r0 - t.a, pbuf, c, [&](int r) { return r < bnd ? xv0 : xv1; });
    release_stage(sm, c);
  }
  mark_stages(sm, c);
  consumer_sync();
  uint16_t* out = P_<uint16_t>(od, MK_P_MRG_OUT);
  for (int lr = c.tid; lr < t.b - t.a; lr += NUM_CONSUMERS)
    out[t.a + lr] = (uint16_t)f32_to_bf16_bits(row_total<KS>(pbuf, lr, ks_of<KS>(DC)));
}

// o_c = (sum over live splits j, in order, of f32(w_j o_j[c])) / (sum of w_j), w_j =
// det_exp(lse_j - max lse); o rounded to BF16; attn rows are row dots with o.
__device__ void merge_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                           Cons& c) {
  const int NH = (int)I_(od, MK_I_MRG_NH), DV = (int)I_(od, MK_I_MRG_DV), DC = (int)I_(od, MK_I_MRG_DC);
  const int S = (int)I_(od, MK_I_MRG_SPLIT), prow = (int)I_(od, MK_I_MRG_PROW);
  const float* partials = P_<const float>(od, MK_P_MRG_PARTIALS);
  const int live = (itx.pos + 1 + S - 1) / S;
  const int hf = t.a / DV, hl = (t.b - 1) / DV;
  const int nh_t = hl - hf + 1;
  uint16_t* obuf = xbuf_of(sm);      // nh_t x DC merged o, BF16
  float* wbuf = pbuf_of(sm);         // nh_t x live: w_j (before the GEMV uses the buffer)
  const size_t jstride = (size_t)NH * prow;
  // a thread owns column quads tid, tid + 256, ...; the first quad's (up to MJ) split values are
  // loaded before anything waits, so they travel together with the lse loads below
  constexpr int MJ = 10;
  const int q4 = DC / 4, nq = nh_t * q4;
  float4 v[MJ];
  if (c.tid < nq) {
    const float* pr = partials + (size_t)(hf + c.tid / q4) * prow + (c.tid % q4) * 4;
#pragma unroll
    for (int u = 0; u < MJ; ++u)
      if (u < live) v[u] = __ldcg(reinterpret_cast<const float4*>(pr + u * jstride));
  }
  if (c.warp < nh_t) {               // one warp per head: M = max lse_j, w_j = det_exp(lse_j - M)
    const float* lse = partials + (size_t)(hf + c.warp) * prow + DC;
    float* wj = wbuf + c.warp * live;
    const float l0 = c.lane < live ? ldcg_f32(lse + c.lane * jstride) : -__int_as_float(0x7F800000);
    float M = l0;
    for (int jj = c.lane + 32; jj < live; jj += 32) M = fmaxf(M, ldcg_f32(lse + jj * jstride));
    M = warp_max_f32(M);
    if (c.lane < live) wj[c.lane] = det_exp(__fsub_rn(l0, M));
    for (int jj = c.lane + 32; jj < live; jj += 32) wj[jj] = det_exp(__fsub_rn(ldcg_f32(lse + jj * jstride), M));
  }
  consumer_sync();
  // o_c = (sum over splits in order of f32(w_j o_j[c])) / (sum over splits in order of w_j)
  for (int quad = c.tid; quad < nq; quad += NUM_CONSUMERS) {
    const int hh = quad / q4, cc = (quad % q4) * 4;
    const float* pr = partials + (size_t)(hf + hh) * prow + cc;
    const float* wj = wbuf + hh * live;
    float n0 = 0.0f, n1 = 0.0f, n2 = 0.0f, n3 = 0.0f, den = 0.0f;
    for (int j0 = 0; j0 < live; j0 += MJ) {
      if (quad != c.tid || j0 != 0) {
#pragma unroll
        for (int u = 0; u < MJ; ++u)
          if (j0 + u < live) v[u] = __ldcg(reinterpret_cast<const float4*>(pr + (j0 + u) * jstride));
      }
#pragma unroll
      for (int u = 0; u < MJ; ++u) {
        if (j0 + u < live) {
          const float w = wj[j0 + u];
          n0 = __fadd_rn(n0, __fmul_rn(w, v[u].x));
          n1 = __fadd_rn(n1, __fmul_rn(w, v[u].y));
          n2 = __fadd_rn(n2, __fmul_rn(w, v[u].z));
          n3 = __fadd_rn(n3, __fmul_rn(w, v[u].w));
          den = __fadd_rn(den, w);
        }
      }
    }
    const uint32_t o0 = f32_to_bf16_bits(__fdiv_rn(n0, den)), o1 = f32_to_bf16_bits(__fdiv_rn(n1, den));
    const uint32_t o2 = f32_to_bf16_bits(__fdiv_rn(n2, den)), o3 = f32_to_bf16_bits(__fdiv_rn(n3, den));
    *reinterpret_cast<uint2*>(obuf + hh * DC + cc) = make_uint2(o0 | (o1 << 16), o2 | (o3 << 16));
  }
  consumer_sync();
  mark_body(sm, c);
  switch (parts_of(DC)) {   // attn rows: row dots with the row's head's o (in shared memory)
    case 2: merge_rows<2>(P, sm, od, t, obuf, hf, DV, DC, c); break;   // D_C 512
    default: merge_rows<0>(P, sm, od, t, obuf, hf, DV, DC, c); break;
  }
}

// ---- router: norm2, FP32 logits, softmax, top-k with the shared experts forced in -----------

// The routing of the last router task to arrive (one warp, E <= 32 EK): softmax over the logits
// (lane l holds experts l, l + 32, ...; max; det_exp; FP32 sum in lane order, then the butterfly;
// one division each), top-k by repeated argmax with ties to the lower index, the forced (shared)
// experts E, E + 1, ... in the last NF slots with weight 1. An argmax round is two warp
// reductions: the maximum of the lanes' best probability bits (non-negative floats order like
// their bit patterns; removed entries are -inf, below them), then the lowest expert index among
// the lanes holding that value.
template <int EK>
__device__ __forceinline__ void route_warp(const KernelParams& P, Smem& sm, const OpDev& od, const Iter itx,
                                        const float* logits, int lane) {
  const int E = (int)I_(od, MK_I_RT_E), TOPK = (int)I_(od, MK_I_RT_TOPK), NF = (int)I_(od, MK_I_RT_NFORCED);
  const float NEG_INF = -__int_as_float(0x7F800000);
  float lv[EK], pv[EK];
  float mx = NEG_INF;
  const uint64_t* ltag = P_<const uint64_t>(od, MK_P_RT_LOGTAG);
  if (ltag) {
    // every task's tagged logits: a word whose tag is this iteration's carries its logit
    bool ok = true;
    const uint64_t t0 = globaltimer();
    // the lane's EK words in flight together, again until each carries this iteration's tag
    uint32_t need = 0u;
#pragma unroll
    for (int k = 0; k < EK; ++k) {
      lv[k] = NEG_INF;
      if (lane + 32 * k < E) need |= 1u << k;
    }
    for (uint32_t n = 0; need; ++n) {
      uint64_t w[EK];
#pragma unroll
      for (int k = 0; k < EK; ++k) w[k] = (need >> k) & 1u ? ld_relaxed_gpu_u64(ltag + lane + 32 * k) : 0u;
#pragma unroll
      for (int k = 0; k < EK; ++k)
        if (((need >> k) & 1u) && (uint32_t)(w[k] >> 32) == itx.g) {
          lv[k] = __uint_as_float((uint32_t)w[k]);
          need &= ~(1u << k);
        }
      if (need && (n & 31u) == 31u && (aborted(P, sm) || (int64_t)(globaltimer() - t0) > P.timeout_ns)) {
        ok = false;
        break;
      }
    }
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0)
        report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_WAIT_TIMEOUT,
                     (uint32_t)od.task0, 0u, 0x30000u | (uint32_t)I_(od, MK_I_RT_LAYER));
      return;
    }
#pragma unroll
    for (int k = 0; k < EK; ++k) mx = fmaxf(mx, lv[k]);
  } else {
#pragma unroll
    for (int k = 0; k < EK; ++k) {
      const int e = lane + 32 * k;
      lv[k] = e < E ? ldcg_f32(logits + e) : NEG_INF;
      mx = fmaxf(mx, lv[k]);
    }
  }
  mx = warp_max_f32(mx);
  float s = 0.0f;   // lane l adds experts l, l + 32, ... in order, then the butterfly
#pragma unroll
  for (int k = 0; k < EK; ++k) {
    const int e = lane + 32 * k;
    pv[k] = e < E ? det_exp(__fsub_rn(lv[k], mx)) : 0.0f;
    if (e < E) s = __fadd_rn(s, pv[k]);
  }
  const float sf = warp_butterfly(s);
#pragma unroll
  for (int k = 0; k < EK; ++k) {
    const int e = lane + 32 * k;
    pv[k] = e < E ? __fdiv_rn(pv[k], sf) : NEG_INF;
  }
  const int ET = E + NF, NSL = TOPK + NF;
  float* topk_w = P_<float>(od, MK_P_RT_TOPKW);
  int32_t* routing = P_<int32_t>(od, MK_P_RT_ROUTING);
  int32_t* mask = P_<int32_t>(od, MK_P_RT_MASK);
  int32_t* rlog = P_<int32_t>(od, MK_P_RT_ROUTELOG);
  for (int e = lane; e < ET; e += 32) routing[e] = 0;
  for (int e = lane; e <= ET; e += 32) mask[e] = -1;
  __syncwarp();
  const float scaling = (float)od.op.fp[1];
  int my_sel = -1;   // lane k < NSL keeps slot k's expert
  for (int k = 0; k < TOPK; ++k) {
    // the lane's best (ties to the lower index; its experts ascend with q)
    float lb = pv[0];
    int li = lane;
#pragma unroll
    for (int q = 1; q < EK; ++q)
      if (pv[q] > lb) { lb = pv[q]; li = lane + 32 * q; }
    const int mb = __reduce_max_sync(0xffffffffu, __float_as_int(lb));
    const int bi = __reduce_min_sync(0xffffffffu, __float_as_int(lb) == mb ? li : 0x7FFFFFFF);
    if (lane == k) my_sel = bi;
    if (lane == 0) topk_w[k] = __fmul_rn(__int_as_float(mb), scaling);
#pragma unroll
    for (int q = 0; q < EK; ++q)
      if (lane + 32 * q == bi) pv[q] = NEG_INF;
  }
  if (lane >= TOPK && lane < NSL) {
    my_sel = E + (lane - TOPK);
    topk_w[lane] = 1.0f;
  }
  __syncwarp();
  if (lane < NSL) {
    routing[my_sel] = lane + 1;
    mask[lane] = my_sel;
    if (uint64_t* mtag = P_<uint64_t>(od, MK_P_RT_MASKTAG))
      st_relaxed_gpu_u64(mtag + lane, ((uint64_t)itx.g << 32) | (uint32_t)my_sel);
    if (rlog) {
      const int layer = (int)I_(od, MK_I_RT_LAYER);
      const int64_t rows = I_(od, MK_I_RT_LOGROWS) > 0 ? I_(od, MK_I_RT_LOGROWS) : 1;
      const int64_t row = (int64_t)((itx.g - 1u) % (uint64_t)rows);
      rlog[row * I_(od, MK_I_RT_LOGSTRIDE) + (int64_t)layer * NSL + lane] = my_sel;
    }
  }
  if (lane == 0) mask[ET] = NSL;
}

template <int KS>
__device__ void router_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                            Cons& c) {
  const int H = (int)I_(od, MK_I_RT_H), E = (int)I_(od, MK_I_RT_E), TOPK = (int)I_(od, MK_I_RT_TOPK),
            NF = (int)I_(od, MK_I_RT_NFORCED);
  uint16_t* hbuf = xbuf_of(sm);
  rmsnorm_to_smem(P_<const uint16_t>(od, MK_P_RT_X), P_<const uint16_t>(od, MK_P_RT_WNORM), H, (float)od.op.fp[0],
                  hbuf, sm, c);
  if (t.idx == 0) {
    uint16_t* hout = P_<uint16_t>(od, MK_P_RT_HOUT);
    for (int i = c.tid; i < H; i += NUM_CONSUMERS) hout[i] = hbuf[i];
  }
  const uint4 xv = x_part<KS, true>(hbuf, H, c);
  mark_body(sm, c);
  float* pbuf = pbuf_of(sm);
  for (int r0 = t.a; r0 < t.b; r0 += od.rps) {
    const int nr = min(od.rps, t.b - r0);
    const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    stage_parts<KS>(stg, nr, H, r0 - t.a, pbuf, c, [&](int) { return xv; });
    release_stage(sm, c);
  }
  consumer_sync();
  float* logits = P_<float>(od, MK_P_RT_LOGITS);
  const float* bias = P_<const float>(od, MK_P_RT_BIAS);
  uint64_t* ltag = P_<uint64_t>(od, MK_P_RT_LOGTAG);
  for (int lr = c.tid; lr < t.b - t.a; lr += NUM_CONSUMERS) {
    float l = row_total<KS>(pbuf, lr, ks_of<KS>(H));
    if (bias) l = __fadd_rn(l, __ldg(bias + t.a + lr));
    logits[t.a + lr] = l;
    if (ltag) st_relaxed_gpu_u64(ltag + t.a + lr, ((uint64_t)itx.g << 32) | __float_as_uint(l));
  }
  if (ltag) {   // task 0 routes from the tagged logits (warp 0); no arrival counter
    mark_stages(sm, c);
    if (t.idx != 0 || c.warp != 0) return;
    if (E <= 64) route_warp<2>(P, sm, od, itx, logits, c.lane);
    else route_warp<8>(P, sm, od, itx, logits, c.lane);
    return;
  }
  consumer_sync();
  if (c.tid == 0) {   // acq_rel: releases the CTA's logits (through the barrier), acquires the others'
    const uint32_t old = atom_add_acqrel(&P.arrive[t.op], 1u);
    sm.bcast[1] = (old + 1u == (uint32_t)od.ntasks * itx.g) ? 1 : 0;
  }
  consumer_sync();
  mark_stages(sm, c);
  if (!sm.bcast[1] || c.warp != 0) return;
  // the last task to arrive routes (one warp; E <= 32 * 8), after thread 0's acquire and the barrier
  (void)TOPK;
  (void)NF;
  if (E <= 64) route_warp<2>(P, sm, od, itx, logits, c.lane);
  else route_warp<8>(P, sm, od, itx, logits, c.lane);
}

// ---- gate-up GEMV with the SwiGLU fused (MoE slots, or layer 0's dense MLP) ------------------
template <int KS>
__device__ void gateup_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                            Cons& c) {
  const int K = (int)I_(od, MK_I_GU_K), I = (int)I_(od, MK_I_GU_I);
  uint4 xv;
  if (od.op.flags & MK_F_NORM) {
    uint16_t* hbuf = xbuf_of(sm);
    rmsnorm_to_smem(P_<const uint16_t>(od, MK_P_GU_X), P_<const uint16_t>(od, MK_P_GU_WNORM), K, (float)od.op.fp[0],
                    hbuf, sm, c);
    uint16_t* hout = P_<uint16_t>(od, MK_P_GU_HOUT);
    if (hout && t.idx == 0)
      for (int i = c.tid; i < K; i += NUM_CONSUMERS) hout[i] = hbuf[i];
    xv = x_part<KS, true>(hbuf, K, c);
  } else {
    xv = x_part<KS, false>(P_<const uint16_t>(od, MK_P_GU_X), K, c);
  }
  (void)itx;
  mark_body(sm, c);
  float* pbuf = pbuf_of(sm);   // [2 * pairs][KS]: local row 2 lp = gate, 2 lp + 1 = up
  const GuMap gm = gu_map(od, t);
  int p = gm.a;
  GuChunk ch;
  while (gu_next(od, p, gm.b, ch)) {
    const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    const int base = (ch.group * I + ch.q) - gm.a;   // local pair index of the chunk's first pair
    stage_parts<KS>(stg, 2 * ch.np, K, 2 * base, pbuf, c, [&](int) { return xv; });
    release_stage(sm, c);
  }
  mark_stages(sm, c);
  consumer_sync();
  uint16_t* act = P_<uint16_t>(od, MK_P_GU_ACT);
  uint16_t* mid = P_<uint16_t>(od, MK_P_GU_MID);
  for (int lp = c.tid; lp < gm.b - gm.a; lp += NUM_CONSUMERS) {
    const int gp = gm.a + lp, g = gu_slot(gm, gp / I), q = gp % I;
    const uint32_t gb = f32_to_bf16_bits(row_total<KS>(pbuf, 2 * lp, ks_of<KS>(K)));
    const uint32_t ub = f32_to_bf16_bits(row_total<KS>(pbuf, 2 * lp + 1, ks_of<KS>(K)));
    const float a = __fmul_rn(det_silu(bf16_bits_to_f32(gb)), bf16_bits_to_f32(ub));
    act[(size_t)g * I + q] = (uint16_t)f32_to_bf16_bits(a);
    if (mid) { mid[(size_t)g * 2 * I + q] = (uint16_t)gb; mid[(size_t)g * 2 * I + I + q] = (uint16_t)ub; }
  }
}

// ---- expert down projection per slot, then the weighted combine into x_res ------------------
// With MK_F_EP the task computes its rank's slots (w2_slots), exchanges the routed rows with the
// same task of every peer rank, and combines all slots of its rows.
template <int KS>
__device__ void w2_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                        Cons& c) {
  const int H = (int)I_(od, MK_I_W2_H), I = (int)I_(od, MK_I_W2_I), NS = (int)I_(od, MK_I_W2_SLOTS);
  const uint16_t* act = P_<const uint16_t>(od, MK_P_W2_ACT);
  const int nr_t = t.b - t.a;
  const bool ep = (od.op.flags & MK_F_EP) != 0;
  const uint32_t wsl = w2_slots(od);   // the slots computed here
  const int wn = __popc(wsl);
  // shared scratch: all slots' activations, the slot weights, the slots' BF16 outputs, partials
  uint16_t* abuf = reinterpret_cast<uint16_t*>(sm.scratch);                         // NS x I
  float* wk = reinterpret_cast<float*>(sm.scratch + w2_aux_off(NS, I));              // NS slot weights
  float* obs = wk + MAX_ROUTED;                                                      // [NS][rows]
  float* pbuf = reinterpret_cast<float*>(sm.scratch + W2_PBUF_OFF);                  // [NS * rows][KS]
  // one round of loads before the stages: the activations (16-byte pieces), the slot weights and
  // each row's residual, so the epilogue waits for no global load
  const float* topk_w = P_<const float>(od, MK_P_W2_TOPKW);
  uint16_t* xres = P_<uint16_t>(od, MK_P_W2_XRES);
  for (int i = c.tid; i < NS * I / 8; i += NUM_CONSUMERS)
    reinterpret_cast<uint4*>(abuf)[i] = ldcg16(act + (size_t)i * 8);
  if (c.tid < NS) wk[c.tid] = ldcg_f32(topk_w + c.tid);
  const float res = c.tid < nr_t ? bf16_bits_to_f32(ldcg_u16(xres + t.a + c.tid)) : 0.0f;
  consumer_sync();
  mark_body(sm, c);
  (void)itx;
  for (uint32_t sl = wsl; sl; sl &= sl - 1u) {
    const int s = __ffs(sl) - 1;
    const uint4 xv = x_part<KS, true>(abuf + (size_t)s * I, I, c);
    for (int r0 = t.a; r0 < t.b; r0 += od.rps) {
      const int nr = min(od.rps, t.b - r0);
      const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
      stage_parts<KS>(stg, nr, I, s * nr_t + (r0 - t.a), pbuf, c, [&](int) { return xv; });
      release_stage(sm, c);
    }
  }
  mark_stages(sm, c);
  consumer_sync();
  // the slots computed here: BF16 outputs, one (slot, row) per thread
  uint16_t* out8 = P_<uint16_t>(od, MK_P_W2_OUT8);
  for (int i = c.tid; i < wn * nr_t; i += NUM_CONSUMERS) {
    const int k = i / nr_t, lr = i - k * nr_t, s = (int)__fns(wsl, 0u, k + 1);
    const uint32_t ob = f32_to_bf16_bits(row_total<KS>(pbuf, s * nr_t + lr, ks_of<KS>(I)));
    obs[s * nr_t + lr] = bf16_bits_to_f32(ob);
    if (out8) out8[(size_t)s * H + t.a + lr] = (uint16_t)ob;
  }
  consumer_sync();
  if (ep) {
    // the slots computed here go to every peer as tagged words (rows 2k, 2k + 1 of a slot per
    // 64-bit word, the iteration's tag in the high half); the other ranks' slots are read from this
    // rank's own words as their tags arrive. The exchange is per task (the same rows on every
    // rank), with no operator boundary, no fence and no counter: a word whose tag is the
    // iteration's carries that iteration's data. The halves alternate by the tag's parity, so a
    // peer overwrites a word only two iterations later, after this rank has sent the next
    // iteration's first exchange, which follows this read.
    const MkEpPeers* pe = P_<const MkEpPeers>(od, MK_P_W2_PEERS);
    const int nranks = pe->nranks, me = pe->rank;
    const uint32_t tag = P.ep_gen0 + (uint32_t)itx.it;
    const size_t hw = (size_t)H / 2;
    const size_t base = ((size_t)(tag & 1u) * (size_t)pe->n_layers + (size_t)I_(od, MK_I_W2_LAYER)) * (size_t)NS * hw +
                        (size_t)(t.a / 2);
    const int npair = nr_t / 2;     // the runtime gives expert-parallel tasks even row ranges
    const int nsend = wn * npair;
    for (int i = c.tid; i < nsend * (nranks - 1); i += NUM_CONSUMERS) {
      const int pi = i % nsend, rr = i / nsend, r = rr < me ? rr : rr + 1;
      const int k = pi / npair, q = pi - k * npair, s = (int)__fns(wsl, 0u, k + 1);
      const uint32_t lo = f32_to_bf16_bits(obs[s * nr_t + 2 * q]), hi = f32_to_bf16_bits(obs[s * nr_t + 2 * q + 1]);
      st_relaxed_sys_u64(pe->xch[r] + base + (size_t)s * hw + q, ((uint64_t)tag << 32) | (uint64_t)(lo | (hi << 16)));
    }
    const uint32_t others = (NS >= 32 ? 0xFFFFFFFFu : (1u << NS) - 1u) & ~wsl;
    const int nrecv = __popc(others) * npair;
    for (int i = c.tid; i < nrecv; i += NUM_CONSUMERS) {
      const int k = i / npair, q = i - k * npair, s = (int)__fns(others, 0u, k + 1);
      const uint64_t* wp = pe->xch[me] + base + (size_t)s * hw + q;
      uint64_t w = ld_relaxed_sys_u64(wp);
      if ((uint32_t)(w >> 32) != tag) {
        const uint64_t t0 = globaltimer();
        bool ok = true;
        for (uint32_t n = 0;; ++n) {
          w = ld_relaxed_sys_u64(wp);
          if ((uint32_t)(w >> 32) == tag) break;
          if ((n & 31u) == 31u && (aborted(P, sm) || (int64_t)(globaltimer() - t0) > P.timeout_ns)) {
            ok = false;
            break;
          }
        }
        if (!ok) {
          report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_WAIT_TIMEOUT,
                       (uint32_t)t.op, (uint32_t)t.idx, 0x20000u | (uint32_t)I_(od, MK_I_W2_LAYER));
          break;
        }
      }
      obs[s * nr_t + 2 * q] = bf16_bits_to_f32((uint32_t)w & 0xFFFFu);
      obs[s * nr_t + 2 * q + 1] = bf16_bits_to_f32(((uint32_t)w >> 16) & 0xFFFFu);
    }
    consumer_sync();
    if (*(volatile uint32_t*)&sm.cta_abort) return;
  }
  for (int lr = c.tid; lr < nr_t; lr += NUM_CONSUMERS) {
    const int row = t.a + lr;
    float acc = lr == c.tid ? res : bf16_bits_to_f32(ldcg_u16(xres + row));
    for (int s = 0; s < NS; ++s)   // numpy_ref.moe_combine's operation order: acc + f32(out * w)
      acc = __fadd_rn(acc, __fmul_rn(obs[s * nr_t + lr], wk[s]));
    xres[row] = (uint16_t)f32_to_bf16_bits(acc);
  }
}

// ---- expert units: gate/up, SwiGLU and the down projection's subtree sums ----------------------
// A task runs its range of units (slot s, part p, lane class q). Per unit: the gate/up rows of
// its intermediates through the row engine (the GATEUP arithmetic: BF16 gate and up, act =
// bf16(silu(gate) up)), then, one row per thread, each of its lanes' down-projection value
// (even products + odd products, the row engine's lane value) and the two butterfly levels over
// the class: S_q = (v_q + v_(q+16)) + (v_(q+8) + v_(q+24)), +0 for lanes without values.
template <int KS, bool FP8>
__device__ void moe_units_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                               Cons& c) {
  const int H = (int)I_(od, MK_I_MU_H), I = (int)I_(od, MK_I_MU_I);
  const int KP = unit_parts(I), Lp = I / KP, l8 = Lp / 8, slot0 = (int)I_(od, MK_I_MU_SLOT0);
  const int r13 = unit_w13_rows((int64_t)H * (FP8 ? 1 : 2));
  uint4 xv;
  if (od.op.flags & MK_F_NORM) {
    uint16_t* hbuf = xbuf_of(sm);
    rmsnorm_to_smem(P_<const uint16_t>(od, MK_P_MU_X), P_<const uint16_t>(od, MK_P_MU_WNORM), H, (float)od.op.fp[0],
                    hbuf, sm, c);
    uint16_t* hout = P_<uint16_t>(od, MK_P_MU_HOUT);
    if (hout && t.idx == 0)
      for (int i = c.tid; i < H; i += NUM_CONSUMERS) hout[i] = hbuf[i];
    xv = x_part<KS, true>(hbuf, H, c);
  } else {
    xv = x_part<KS, false>(P_<const uint16_t>(od, MK_P_MU_X), H, c);
  }
  if constexpr (FP8) xv = bf16x8_to_f16x8(xv);   // the FP8 products take FP16 activations
  (void)itx;
  mark_body(sm, c);
  float* pbuf = pbuf_of(sm);
  uint16_t* abuf = reinterpret_cast<uint16_t*>(sm.scratch + MU_ABUF_OFF);
  float* sums = P_<float>(od, MK_P_MU_SUMS);
  uint16_t* actg = P_<uint16_t>(od, MK_P_MU_ACT);
  const float* s13 = P_<const float>(od, MK_P_MU_SCALE13);
  const MuList ml = mu_list(t);
  for (int v = 0; v < ml.nf + ml.nr; ++v) {   // the fixed slots' units, then the routed slots'
    const int u = P.units[ml.off + v];
    const int s = slot0 + u / (KP * 8), pt = (u >> 3) % KP, q = u & 7, nl = unit_lanes(q, l8);
    float sg = 1.0f, su = 1.0f;   // FP8: the unit's expert's gate and up scales
    for (int j = 0; j < nl; ++j)
      for (int r = 0; r < 16; r += r13) {
        const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
        if constexpr (FP8) {
          if (j == 0 && r == 0 && c.tid < 8 * nl) {   // the expert the producer attached to the stage
            const int e = sm.stage_aux[(c.c_it - 1) % NSTAGES];
            sg = __ldg(s13 + 2 * e);
            su = __ldg(s13 + 2 * e + 1);
          }
          stage_parts_fp8<KS>(stg, r13, H, 16 * j + r, pbuf, c, xv);
        } else {
          stage_parts<KS>(stg, r13, H, 16 * j + r, pbuf, c, [&](int) { return xv; });
        }
        release_stage(sm, c);
      }
    consumer_sync();
    if (c.tid < 8 * nl) {   // intermediate 8 (q + 8 j) + k of the part: local rows 16 j + 2 k (gate), + 1 (up)
      const int j = c.tid >> 3, k = c.tid & 7;
      float gt = row_total<KS>(pbuf, 16 * j + 2 * k, ks_of<KS>(H));
      float ut = row_total<KS>(pbuf, 16 * j + 2 * k + 1, ks_of<KS>(H));
      if constexpr (FP8) {
        gt = __fmul_rn(sg, gt);
        ut = __fmul_rn(su, ut);
      }
      const uint32_t gb = f32_to_bf16_bits(gt), ub = f32_to_bf16_bits(ut);
      const uint32_t ab = f32_to_bf16_bits(__fmul_rn(det_silu(bf16_bits_to_f32(gb)), bf16_bits_to_f32(ub)));
      abuf[c.tid] = (uint16_t)ab;
      if (actg) actg[(size_t)s * I + pt * Lp + 8 * (q + 8 * j) + k] = (uint16_t)ab;
    }
    consumer_sync();
    const uint32_t ab0 = smem_u32(abuf);
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    uint4 x0 = lds128(ab0), x1 = nl > 1 ? lds128(ab0 + 16u) : z, x2 = nl > 2 ? lds128(ab0 + 32u) : z,
          x3 = nl > 3 ? lds128(ab0 + 48u) : z;
    if constexpr (FP8) {
      x0 = bf16x8_to_f16x8(x0);
      x1 = bf16x8_to_f16x8(x1);
      x2 = bf16x8_to_f16x8(x2);
      x3 = bf16x8_to_f16x8(x3);
    }
    float* out = sums + ((size_t)(s * KP + pt) * 8 + q) * H;
    constexpr int LB = FP8 ? 8 : 16;   // bytes of a lane's eight weights
    const int rb = LB * nl, r2 = unit_w2_rows(rb);
    for (int r0 = 0; r0 < H; r0 += r2) {
      const int nr = min(r2, H - r0);
      const uint32_t sb = smem_u32(acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx));
      for (int r = c.tid; r < nr; r += NUM_CONSUMERS) {
        const uint32_t ra = sb + (uint32_t)(r * rb);
        auto lane_value = [&](uint32_t a, const uint4& x) {
          if constexpr (FP8) {
            return lane_fp8(lds64(a), x);
          } else {
            const uint4 w = lds128(a);
            float a0 = 0.0f, a1 = 0.0f;
            fma_bf16x2(a0, a1, w.x, x.x);
            fma_bf16x2(a0, a1, w.y, x.y);
            fma_bf16x2(a0, a1, w.z, x.z);
            fma_bf16x2(a0, a1, w.w, x.w);
            return __fadd_rn(a0, a1);
          }
        };
        const float v0 = lane_value(ra, x0);
        const float v1 = nl > 1 ? lane_value(ra + LB, x1) : 0.0f;
        const float v2 = nl > 2 ? lane_value(ra + 2 * LB, x2) : 0.0f;
        const float v3 = nl > 3 ? lane_value(ra + 3 * LB, x3) : 0.0f;
        out[r0 + r] = __fadd_rn(__fadd_rn(v0, v2), __fadd_rn(v1, v3));
      }
      release_stage(sm, c);
    }
  }
  mark_stages(sm, c);
}

// ---- expert combine: the down projection per slot from the subtree sums, then x += sum w out8 --
// One (slot, part, row) per thread for the part sums (the butterfly's last three levels), then
// one (slot, row) per thread for the parts in order and the BF16 rounding, then the combine of
// numpy_ref.moe_combine (acc + f32(out * w) in slot order).
__device__ void moe_combine_body(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                                 Cons& c) {
  const int H = (int)I_(od, MK_I_MC_H), I = (int)I_(od, MK_I_MC_I), NS = (int)I_(od, MK_I_MC_NS);
  const int KP = unit_parts(I), l8 = (I / KP) / 8, nr = t.b - t.a;
  const float* sums = P_<const float>(od, MK_P_MC_SUMS);
  const float* topk_w = P_<const float>(od, MK_P_MC_TOPKW);
  uint16_t* xres = P_<uint16_t>(od, MK_P_MC_XRES);
  uint16_t* out8 = P_<uint16_t>(od, MK_P_MC_OUT8);
  float* psum = reinterpret_cast<float*>(sm.scratch);       // [NS][KP][nr]
  float* obs = psum + NS * KP * nr;                          // [NS][nr]
  float* wk = obs + NS * nr;                                 // [NS]
  (void)itx;
  (void)P;
  float* dsc = wk + NS;                                       // [NS] FP8: the slots' down scales
  if (c.tid < NS) {
    wk[c.tid] = ldcg_f32(topk_w + c.tid);
    if (od.op.flags & MK_F_FP8)
      dsc[c.tid] = __ldg(P_<const float>(od, MK_P_MC_SCALE2) + __ldcg(P_<const int32_t>(od, MK_P_MC_MASK) + c.tid));
  }
  const float res = c.tid < nr ? bf16_bits_to_f32(ldcg_u16(xres + t.a + c.tid)) : 0.0f;
  mark_body(sm, c);
  bool live[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) live[q] = unit_lanes(q, l8) > 0;
  const int n = NS * KP * nr;
  constexpr int NB = 4;   // four items' loads in flight at a time (one round at the model's sizes)
  for (int i0 = c.tid; i0 < n; i0 += NB * NUM_CONSUMERS) {
    float S[NB][8];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int i = i0 + k * NUM_CONSUMERS;
      const int lr = i % nr, sp = i / nr;
      const float* src = sums + (size_t)sp * 8 * H + t.a + lr;
#pragma unroll
      for (int q = 0; q < 8; ++q) S[k][q] = (i < n && live[q]) ? __ldcg(src + (size_t)q * H) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int i = i0 + k * NUM_CONSUMERS;
      if (i < n)
        psum[i] = __fadd_rn(__fadd_rn(__fadd_rn(S[k][0], S[k][4]), __fadd_rn(S[k][2], S[k][6])),
                            __fadd_rn(__fadd_rn(S[k][1], S[k][5]), __fadd_rn(S[k][3], S[k][7])));
    }
  }
  consumer_sync();
  for (int i = c.tid; i < NS * nr; i += NUM_CONSUMERS) {
    const int s = i / nr, lr = i - s * nr;
    float d = psum[(s * KP) * nr + lr];
    for (int pt = 1; pt < KP; ++pt) d = __fadd_rn(d, psum[(s * KP + pt) * nr + lr]);
    if (od.op.flags & MK_F_FP8) d = __fmul_rn(dsc[s], d);
    const uint32_t ob = f32_to_bf16_bits(d);
    obs[s * nr + lr] = bf16_bits_to_f32(ob);
    if (out8) out8[(size_t)s * H + t.a + lr] = (uint16_t)ob;
  }
  consumer_sync();
  for (int lr = c.tid; lr < nr; lr += NUM_CONSUMERS) {
    float acc = lr == c.tid ? res : bf16_bits_to_f32(ldcg_u16(xres + t.a + lr));
    for (int s = 0; s < NS; ++s) acc = __fadd_rn(acc, __fmul_rn(obs[s * nr + lr], wk[s]));
    xres[t.a + lr] = (uint16_t)f32_to_bf16_bits(acc);
  }
  mark_stages(sm, c);
}

// ---- stream probe: the ring's bytes, no arithmetic -------------------------------------------
__device__ void op_stream(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                          Cons& c) {
  uint32_t x = 0;
  (void)itx;
  for (int r0 = t.a; r0 < t.b; r0 += od.rps) {
    const uint8_t* stg = acquire_stage(P, sm, c, (uint32_t)t.op, (uint32_t)t.idx);
    x ^= reinterpret_cast<const uint32_t*>(stg)[c.tid];
    release_stage(sm, c);
  }
  uint32_t* out = P_<uint32_t>(od, MK_P_ST_OUT);
  if (out && x == 0x9E3779B9u) out[t.idx] = x;   // keeps the read; practically never stores
}

// =============================================================================================
// consumer loop
// =============================================================================================

// Two instantiations per operator (the unrolled 8-part path and a run-time part count): few code
// paths keep the task loop's register allocation and the instruction working set small.
template <int N>
struct PartsTag {
  static constexpr int value = N;
};
template <class F>
__device__ __forceinline__ void by_parts(int K, F&& f) {
  if (parts_of(K) == 8) f(PartsTag<8>{});   // the model's K (2,048 and 1,408): unrolled
  else f(PartsTag<0>{});                    // every other K: run-time part count
}
// Kernel variants: KV_SHORT (the exact attention, one head per task), KV_LONG (adds the exact
// attention's two-heads-at-a-time form, used by head groups > 1 at long context), KV_TC (the
// tensor-core attention instead of both). A plan's launches use the one variant that has its
// operators, so the other forms' code does not sit in the hot kernel.
enum { KV_SHORT = 0, KV_LONG = 1, KV_TC = 2 };
template <int KV>
__device__ void run_task(const KernelParams& P, Smem& sm, const OpDev& od, const TaskDev& t, const Iter& itx,
                         Cons& c) {
  switch (od.op.type) {
    case MK_OP_EMBED: op_embed(P, sm, od, t, itx, c); break;
    case MK_OP_GEMV: {
      const int K = (int)I_(od, MK_I_GEMV_K);
      if (od.ksplit > 1) gemv_wide_body<6>(P, sm, od, t, itx, c);
      else by_parts(K, [&](auto ks) { gemv_body<decltype(ks)::value>(P, sm, od, t, itx, c); });
      break;
    }
    case MK_OP_MLA_PREP: op_prep(P, sm, od, t, itx, c); break;
    case MK_OP_MLA_ATTEND: {
      if constexpr (KV == KV_TC) {
        if (od.op.flags & MK_F_TC) {
          attend_tc(P, sm, od, t, itx, c);
          break;
        }
      }
      if (I_(od, MK_I_ATT_DC) == 512 && I_(od, MK_I_ATT_DR) == 64) {
        if constexpr (KV == KV_LONG) {
          if ((I_(od, MK_I_ATT_HGROUP) & 1) == 0) {
            attend_pairs(P, sm, od, t, itx, c);
            break;
          }
        }
        attend_body<true>(P, sm, od, t, itx, c);
      }
      else attend_body<false>(P, sm, od, t, itx, c);
      break;
    }
    case MK_OP_MLA_MERGE_UV: merge_body(P, sm, od, t, itx, c); break;
    case MK_OP_ROUTER: {
      const int H = (int)I_(od, MK_I_RT_H);
      by_parts(H, [&](auto ks) { router_body<decltype(ks)::value>(P, sm, od, t, itx, c); });
      break;
    }
    case MK_OP_GATEUP: {
      const int K = (int)I_(od, MK_I_GU_K);
      by_parts(K, [&](auto ks) { gateup_body<decltype(ks)::value>(P, sm, od, t, itx, c); });
      break;
    }
    case MK_OP_W2_COMBINE: {
      const int I = (int)I_(od, MK_I_W2_I);
      by_parts(I, [&](auto ks) { w2_body<decltype(ks)::value>(P, sm, od, t, itx, c); });
      break;
    }
    case MK_OP_STREAM: op_stream(P, sm, od, t, itx, c); break;
    case MK_OP_COPY: op_copy(od, c); break;
    case MK_OP_MOE_UNITS: {
      const int H = (int)I_(od, MK_I_MU_H);
      if (od.op.flags & MK_F_FP8) by_parts(H, [&](auto ks) { moe_units_body<decltype(ks)::value, true>(P, sm, od, t, itx, c); });
      else by_parts(H, [&](auto ks) { moe_units_body<decltype(ks)::value, false>(P, sm, od, t, itx, c); });
      break;
    }
    case MK_OP_MOE_COMBINE: moe_combine_body(P, sm, od, t, itx, c); break;
    default: break;
  }
}

// The next task's list entry and operator descriptor are copied into shared memory (cp.async)
// while the current task runs, so a task starts without a global round trip for them.
constexpr int OPDEV_CHUNKS = (int)(sizeof(OpDev) / 16);
__device__ __forceinline__ void prefetch_task(const KernelParams& P, Smem& sm, uint32_t k, int op, int slot,
                                              int tid) {
  if (tid < OPDEV_CHUNKS)
    cp_async16(reinterpret_cast<uint4*>(&sm.od_buf[slot]) + tid, reinterpret_cast<const uint4*>(P.ops + op) + tid);
  else if (tid < OPDEV_CHUNKS + 2)
    cp_async16(reinterpret_cast<uint4*>(&sm.ct_buf[slot]) + (tid - OPDEV_CHUNKS),
               reinterpret_cast<const uint4*>(P.ctask + k) + (tid - OPDEV_CHUNKS));
}

template <int KV>
__device__ void consumer_main(const KernelParams& P, Smem& sm) {
  Cons c;
  c.c_it = 0u;
  c.c_rel = 0u;
  c.tid = threadIdx.x;
  c.warp = c.tid >> 5;
  c.lane = c.tid & 31;
  c.trace = P.trace != nullptr;
  const uint32_t b = P.cta_off[blockIdx.x], e = P.cta_off[blockIdx.x + 1];
  if (b == e) return;
  prefetch_task(P, sm, b, P.ctask[b].t.op, 0, c.tid);
  cp_async_wait_all();
  consumer_sync();
  int slot = 0;
#pragma unroll 1
  for (int it = 0; it < P.iters; ++it) {
#pragma unroll 1
    for (uint32_t k = b; k < e; ++k, slot ^= 1) {
      // only the loop position and the ring counters stay in registers across the task body
      {
        const TaskDev t = sm.ct_buf[slot].t;
        const OpDev& od = sm.od_buf[slot];
        const uint32_t g = P.gen0 + (uint32_t)it;
        if (it + 1 < P.iters || k + 1 < e)   // the CTA's next task (wrapping to the next iteration)
          prefetch_task(P, sm, k + 1 < e ? k + 1 : b, sm.ct_buf[slot].next_op, slot ^ 1, c.tid);
        if (c.tid == 0) {
          int ok = 1;
          if (*(volatile uint32_t*)&sm.cta_abort) ok = 0;
          for (int j = 0; j < 2 && ok; ++j) {
            const int dep = od.dep_op[j];
            if (dep < 0) continue;
            const uint32_t target = (uint32_t)od.dep_n[j] * (g - (uint32_t)od.dep_lag[j]);
            if (!wait_event(P, sm, &P.events[dep], target, t.op == P.block_op)) {
              report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_WAIT_TIMEOUT,
                           (uint32_t)t.op, (uint32_t)t.idx, (uint32_t)dep);
              ok = 0;
            }
          }
          sm.bcast[0] = ok;
          if (c.trace) { sm.tr[TR_READY] = globaltimer(); sm.tr[TR_BODY] = 0; sm.tr[TR_STAGES] = 0; sm.tr[TR_WAIT] = 0; }
        }
      }
      consumer_sync();
      if (!sm.bcast[0]) goto done;
      {
        const Iter itx{it, P.step + 1 + it, P.gen0 + (uint32_t)it};
        run_task<KV>(P, sm, sm.od_buf[slot], sm.ct_buf[slot].t, itx, c);
      }
      cp_async_wait_all();
      consumer_sync();
      if (c.tid == 0) {
        const TaskDev t = sm.ct_buf[slot].t;
        // a run of tasks of one operator on this CTA (long-context attention) signals once, after
        // its last task (the host's count): one release fence instead of one per task. No task of
        // the run waits for the operator itself, so the deferred count cannot hold anything up.
        const int sig = sm.ct_buf[slot].signal;
        if (sig && !*(volatile uint32_t*)&sm.cta_abort) red_release_add(&P.events[t.op], (uint32_t)sig);
        if (c.trace) {
          const uint32_t tslot = atomicAdd(P.trace_count, 1u);
          if (tslot < P.trace_cap) {
            MkTraceRecord rec;
            rec.op = (uint32_t)t.op; rec.task = (uint32_t)t.idx; rec.cta = blockIdx.x; rec.iter = (uint32_t)it;
            rec.t_ready = sm.tr[TR_READY]; rec.t_end = globaltimer();
            rec.t_body = sm.tr[TR_BODY]; rec.t_stages = sm.tr[TR_STAGES]; rec.wait_ns = sm.tr[TR_WAIT];
            P.trace[tslot] = rec;
          }
        }
      }
    }
  }
done:
  cp_async_wait_all();
  if (c.tid == 0 && *(volatile uint32_t*)&sm.cta_abort) atomicAdd(&P.status->aborted_ctas, 1u);
}

// One instantiation per kernel variant (KV_SHORT, KV_LONG, KV_TC; see run_task).
template <int KV>
__global__ void __launch_bounds__(NUM_THREADS, 1) mk_persistent_kernel(const KernelParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGES; ++s) {
      mbar_init(&sm.full[s], 1u);
      mbar_init(&sm.empty[s], (uint32_t)NUM_CONSUMER_WARPS);
    }
    sm.cta_abort = 0u;
    fence_barrier_init();
    sm.kp = P;
  }
  __syncthreads();
  // the loops read the parameters from shared memory: the compiler then reloads them where they
  // are used instead of hoisting them into registers that stay live across every operator
  if (threadIdx.x >= NUM_CONSUMERS) {
    if (threadIdx.x == NUM_CONSUMERS) producer_main(sm.kp, sm);
    return;
  }
  consumer_main<KV>(sm.kp, sm);
}

}  // namespace mk
