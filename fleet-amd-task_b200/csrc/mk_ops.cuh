// mk_ops.cuh -- the task kernels of the decode graph, as device functions of the persistent
// kernel. Each operator type has a producer half (which global bytes its tasks stream through
// the shared-memory ring, issued by the producer warp) and a consumer half (what the eight
// consumer warps compute from those stages and from activations in L2).
//
// Arithmetic contract (oracle/numpy_ref.py is the CPU statement of it): every sum is FP32 in the
// order oracle/detmath.py specifies (row dot, butterfly, block / lane / sequential sums); every
// exp/log is det_exp/det_log; the rounding points are the reference's (harness/numpy_ref.py:36-321).
#pragma once
#include "mk_device.cuh"

namespace mk {

// ---- per-launch iteration context ----------------------------------------------------------

struct Iter {
  int32_t it;       // iteration within this launch
  int32_t pos;      // decode position (cache row written, token read)
  uint32_t g;       // global generation (1-based)
};

struct Cons {       // consumer-side state
  uint32_t c_it, c_rel;
  int warp, lane, tid;
  bool trace;                           // record the task stamps in Smem::tr (thread 0 only)
};

// trace stamps of the task body: activations loaded / last weight stage consumed
__device__ __forceinline__ void mark_body(Smem& sm, const Cons& c) {
  if (c.trace && c.tid == 0) sm.tr[TR_BODY] = globaltimer();
}
__device__ __forceinline__ void mark_stages(Smem& sm, const Cons& c) {
  if (c.trace && c.tid == 0) sm.tr[TR_STAGES] = globaltimer();
}

// ---- error reporting ------------------------------------------------------------------------

__device__ __noinline__ void report_error(const KernelParams& P, Smem& sm, uint32_t code, uint32_t op,
                                          uint32_t task, uint32_t info) {
  if (atomicCAS(&P.status->error, 0u, code) == 0u) {
    P.status->err_op = op;
    P.status->err_task = task;
    P.status->err_cta = blockIdx.x;
    P.status->err_info = info;
    __threadfence();
  }
  atomicExch(&P.status->abort_flag, 1u);
  *(volatile uint32_t*)&sm.cta_abort = 1u;
}

__device__ __forceinline__ bool aborted(const KernelParams& P, Smem& sm) {
  return *(volatile uint32_t*)&sm.cta_abort || *(volatile uint32_t*)&P.status->abort_flag;
}

// Bounded spin until *ev >= target (wrap-safe). `never` models the debug hook (an event that
// never fires). Returns false on timeout or when another CTA has aborted.
__device__ __forceinline__ bool wait_event(const KernelParams& P, Smem& sm, const uint32_t* ev, uint32_t target,
                                        bool never) {
  if (!never && (int32_t)(ld_acquire_u32(ev) - target) >= 0) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t n = 1;; ++n) {
    if (!never && (int32_t)(ld_acquire_u32(ev) - target) >= 0) return true;
    if ((n & 31u) == 0u) {
      if (aborted(P, sm)) return false;
      if ((int64_t)(globaltimer() - t0) > P.timeout_ns) return false;
    }
  }
}

// Bounded wait on a ring mbarrier phase.
__device__ __forceinline__ bool ring_wait(const KernelParams& P, Smem& sm, uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 7u) == 0u) {
      if (aborted(P, sm)) return false;
      if ((int64_t)(globaltimer() - t0) > P.timeout_ns) return false;
    }
  }
}

// ---- consumer ring access -------------------------------------------------------------------

__device__ __forceinline__ uint8_t* acquire_stage(const KernelParams& P, Smem& sm, Cons& c, uint32_t op,
                                                  uint32_t task) {
  const uint32_t st = c.c_it % NSTAGES, ph = (c.c_it / NSTAGES) & 1u;
  const uint64_t t0 = (c.trace && c.tid == 0) ? globaltimer() : 0;
  if (!mbar_try_wait(&sm.full[st], ph) && !*(volatile uint32_t*)&sm.cta_abort &&
      !ring_wait(P, sm, &sm.full[st], ph)) {
    if (c.lane == 0)
      report_error(P, sm, *(volatile uint32_t*)&P.status->abort_flag ? MK_DERR_ABORTED : MK_DERR_RING_TIMEOUT,
                   op, task, 1);
  }
  if (c.trace && c.tid == 0) sm.tr[TR_WAIT] += globaltimer() - t0;
  c.c_it++;
  return sm.ring[st];
}
__device__ __forceinline__ uint8_t* stage_ptr(Smem& sm, uint32_t index) { return sm.ring[index % NSTAGES]; }
__device__ __forceinline__ void release_stage(Smem& sm, Cons& c) {
  const uint32_t st = c.c_rel % NSTAGES;
  c.c_rel++;
  __syncwarp();
  if (c.lane == 0) mbar_arrive(&sm.empty[st]);
}

// ---- FP32 dot products in the specified order -------------------------------------------------

// x for vectors v = lane + 32 j of a K-slice, kept as packed BF16 (8 values per uint4: half the
// registers of FP32, unpacked exactly as the products are formed); x is BF16 bits.
template <int MAXV, bool SMEM>
__device__ __forceinline__ void load_x(uint4 (&xr)[MAXV], const uint16_t* x, int klen, int lane) {
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = lane + 32 * j;
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (v * 8 < klen) raw = SMEM ? lds128(smem_u32(x + v * 8)) : ldcg16(x + v * 8);
    xr[j] = raw;
  }
}

// FP32 row dot in the specified order: lane l takes the 8-value vectors l + 32 j (j ascending),
// even values into a0 and odd values into a1, then a0 + a1 and the butterfly. row is in shared
// memory (a weight stage).
template <int MAXV>
__device__ __forceinline__ float row_dot(const uint4 (&xr)[MAXV], const uint8_t* row, int klen, int lane) {
  float a0 = 0.0f, a1 = 0.0f;
  const uint32_t sa = smem_u32(row);
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = lane + 32 * j;
    if (v * 8 < klen) {
      const uint4 w = lds128(sa + v * 16);
      const uint4 x = xr[j];
      fma_bf16x2(a0, a1, w.x, x.x);
      fma_bf16x2(a0, a1, w.y, x.y);
      fma_bf16x2(a0, a1, w.z, x.z);
      fma_bf16x2(a0, a1, w.w, x.w);
    }
  }
  return warp_butterfly(__fadd_rn(a0, a1));
}

// Warp maximum of finite or infinite FP32 values as one integer reduction: the key flips the
// magnitude bits of negative values, so signed keys order like the values (a -0 / +0 tie may
// come back as either zero, which no caller distinguishes: they subtract the maximum).
__device__ __forceinline__ float warp_max_f32(float a) {
  const int b = __float_as_int(a);
  const int m = __reduce_max_sync(0xffffffffu, b >= 0 ? b : b ^ 0x7FFFFFFF);
  return __int_as_float(m >= 0 ? m : m ^ 0x7FFFFFFF);
}

// ---- RMSNorm of a BF16 row into shared memory (all 256 consumer threads) ----------------------
// h = bf16(w * bf16(x * r)), r = 1 / sqrt(ss / K + eps)   (numpy_ref.py:54-60), with ss the FP32
// sum of squares in the block order: thread t adds the 8-value vectors t, t + 256, ... in order,
// the warps reduce by the butterfly, and warps 0..7 are added in order (oracle detmath.block_sum).
constexpr int NORM_MAX_VECS = 2;   // K <= 4096
__device__ void rmsnorm_to_smem(const uint16_t* x, const uint16_t* w, int K, float eps, uint16_t* hbuf, Smem& sm,
                                const Cons& c) {
  // one pass over global memory: a thread's 16-byte vectors are loaded together
  const int nv = K / 8;
  uint4 xv[NORM_MAX_VECS], wv[NORM_MAX_VECS];
#pragma unroll
  for (int k = 0; k < NORM_MAX_VECS; ++k) {
    const int v = c.tid + k * NUM_CONSUMERS;
    xv[k] = v < nv ? ldcg16(x + (size_t)v * 8) : make_uint4(0u, 0u, 0u, 0u);
    wv[k] = v < nv ? __ldg(reinterpret_cast<const uint4*>(w) + v) : make_uint4(0u, 0u, 0u, 0u);
  }
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < NORM_MAX_VECS; ++k) {
    if (c.tid + k * NUM_CONSUMERS < nv) {
      const uint32_t u[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) ss = fma_bf16x2_seq(ss, u[q], u[q]);
    }
  }
  ss = warp_butterfly(ss);
  float* red = reinterpret_cast<float*>(sm.red);
  if (c.lane == 0) red[c.warp] = ss;
  consumer_sync();
  float tot = red[0];
#pragma unroll
  for (int k = 1; k < NUM_CONSUMER_WARPS; ++k) tot = __fadd_rn(tot, red[k]);
  const float var = __fdiv_rn(tot, (float)K);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  auto nrm = [&](float xe, float we) -> uint32_t { return f32_to_bf16_bits(__fmul_rn(we, round_bf16(__fmul_rn(xe, r)))); };
#pragma unroll
  for (int k = 0; k < NORM_MAX_VECS; ++k) {
    const int v = c.tid + k * NUM_CONSUMERS;
    if (v < nv) {
      const uint32_t ux[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
      const uint32_t uw[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o[q] = nrm(lo_f32(ux[q]), lo_f32(uw[q])) | (nrm(hi_f32(ux[q]), hi_f32(uw[q])) << 16);
      reinterpret_cast<uint4*>(hbuf)[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  consumer_sync();   // hbuf complete; sm.red free again
}

// RoPE of one d-vector (de-interleaved pairs; numpy_ref.py:63-71): element i of the output.
__device__ __forceinline__ uint16_t rope_elem(const uint16_t* x, const uint16_t* cosr, const uint16_t* sinr, int d,
                                              int i, bool x_global) {
  const int h = d / 2;
  auto ld = [&](int k) -> float { return bf16_bits_to_f32(x_global ? ldcg_u16(x + k) : (uint32_t)x[k]); };
  const float xi = (i < h) ? ld(2 * i) : ld(2 * (i - h) + 1);
  const float rot = (i < h) ? -ld(2 * i + 1) : ld(2 * (i - h));
  const float cs = bf16_bits_to_f32(__ldg(cosr + i)), sn = bf16_bits_to_f32(__ldg(sinr + i));
  const float a = round_bf16(__fmul_rn(xi, cs));
  const float b = round_bf16(__fmul_rn(rot, sn));
  return (uint16_t)f32_to_bf16_bits(__fadd_rn(a, b));
}

// ---- helpers on operator parameters --------------------------------------------------------

template <typename T>
__device__ __forceinline__ T* P_(const OpDev& od, int i) { return reinterpret_cast<T*>(od.op.ptr[i]); }
__device__ __forceinline__ int64_t I_(const OpDev& od, int i) { return od.op.ip[i]; }

// GATEUP: the stages of a task walk its pair range in chunks inside one group.
struct GuChunk { int group, q, np; };
__device__ __forceinline__ bool gu_next(const OpDev& od, int& p, int b, GuChunk& ch) {
  if (p >= b) return false;
  const int I = (int)I_(od, MK_I_GU_I);
  const int g = p / I, q = p % I;
  int np = od.rps / 2;
  np = min(np, I - q);
  np = min(np, b - p);
  ch.group = g; ch.q = q; ch.np = np;
  p += np;
  return true;
}

// GATEUP: the slot map and pair range of a task. Without MK_F_EP: group g is slot g, the host's
// range. With MK_F_EP (slot parallelism over N ranks): the groups g whose slot SLOT0 + g has
// (SLOT0 + g) mod N = rank, in group order (group g is the g-th set bit of `slots`), and the
// task's share of their pairs (none when the rank has no such group). Slot sets are bit masks,
// not arrays: a dynamically indexed array would live in local memory, whose lines miss the small
// L1 left beside the shared-memory carveout.
struct GuMap { uint32_t slots; int a, b; };
__device__ __forceinline__ int gu_slot(const GuMap& m, int g) { return m.slots ? (int)__fns(m.slots, 0u, g + 1) : g; }
// the groups g < n whose slot s0 + g has (s0 + g) mod world = rank
__device__ __forceinline__ uint32_t rank_slots(int n, int s0, int rank, int world) {
  uint32_t m = 0;
  for (int g = 0; g < n; ++g)
    if ((s0 + g) % world == rank) m |= 1u << g;
  return m;
}
__device__ __forceinline__ GuMap gu_map(const OpDev& od, const TaskDev& t) {
  if (!(od.op.flags & MK_F_EP)) return GuMap{0u, t.a, t.b};
  const int G = (int)I_(od, MK_I_GU_GROUPS), I = (int)I_(od, MK_I_GU_I);
  const uint32_t slots = rank_slots(G, (int)I_(od, MK_I_GU_SLOT0), (int)I_(od, MK_I_GU_EPRANK),
                                    (int)I_(od, MK_I_GU_EPWORLD));
  const int64_t Pn = (int64_t)__popc(slots) * I, T = od.ntasks;
  GuMap m;
  m.slots = slots ? slots : 1u << 31;   // a non-zero set, so the map is not the identity
  m.a = (int)((int64_t)t.idx * Pn / T);
  m.b = (int)((int64_t)(t.idx + 1) * Pn / T);
  return m;
}

// W2_COMBINE: the slots a rank computes, as a bit set in slot order (all, or with MK_F_EP the
// slots s with s mod N = rank, shared slots included).
__device__ __forceinline__ uint32_t w2_slots(const OpDev& od) {
  const int NS = (int)I_(od, MK_I_W2_SLOTS);
  const uint32_t all = NS >= 32 ? 0xFFFFFFFFu : (1u << NS) - 1u;
  if (!(od.op.flags & MK_F_EP)) return all;
  return rank_slots(NS, 0, (int)I_(od, MK_I_W2_EPRANK), (int)I_(od, MK_I_W2_EPWORLD));
}

// MOE_UNITS: a task's units are entries [off, off + nf + nr) of the unit table, the fixed slots'
// nf first, then the routed slots' nr (TaskDev.a = off, TaskDev.b = nf | nr << 16).
struct MuList { int off, nf, nr; };
__device__ __forceinline__ MuList mu_list(const TaskDev& t) { return MuList{t.a, t.b & 0xFFFF, (t.b >> 16) & 0xFFFF}; }

// ATTEND: the split a task covers at this iteration.
struct AttSplit { int lo, hi, n_str, has_pos; };
__device__ __forceinline__ AttSplit att_split(const OpDev& od, const TaskDev& t, int pos) {
  const int S = (int)I_(od, MK_I_ATT_SPLIT);
  AttSplit a;
  a.lo = t.b * S;
  a.hi = min(a.lo + S, pos + 1);
  a.n_str = max(0, min(a.lo + S, pos) - a.lo);
  a.has_pos = (pos >= a.lo && pos < a.lo + S) ? 1 : 0;
  if (a.lo > pos) { a.hi = a.lo; a.n_str = 0; a.has_pos = 0; }
  return a;
}
__device__ __forceinline__ int att_rps(const OpDev& od) {
  return STAGE_BYTES / (int)((I_(od, MK_I_ATT_DC) + I_(od, MK_I_ATT_DR)) * 2);
}

}  // namespace mk
