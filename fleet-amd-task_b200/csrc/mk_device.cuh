// mk_device.cuh -- device-side building blocks of the persistent decode kernel: PTX wrappers
// (mbarriers, bulk copies, release/acquire events, %globaltimer), the shared-memory layout,
// and the tables the host uploads (operators, tasks, per-CTA task lists).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/fleet_mk.h"
#include "detmath.cuh"

namespace mk {

constexpr int NUM_CONSUMER_WARPS = 8;
constexpr int NUM_CONSUMERS = NUM_CONSUMER_WARPS * 32;
constexpr int NUM_THREADS = NUM_CONSUMERS + 32;          // + one producer warp
constexpr int STAGE_BYTES = 32768;
constexpr int NSTAGES = 6;
constexpr int SCRATCH_BYTES = 32768;
constexpr int XBUF_BYTES = 8192;                         // scratch [0, 8 KB): a staged x row
constexpr int PBUF_OFF = XBUF_BYTES;                       // scratch [8 KB, 32 KB): per-task partial sums
constexpr int W2_PBUF_OFF = 24576;                         // the expert down projection stages all slots'
                                                           // activations in [0, 24 KB), partials after
constexpr int MAX_ROUTED = 16;                           // N_SLOTS bound (8 at DeepSeek-V2-Lite)
// expert units: a unit's activations (at most 4 lanes x 8 values, BF16) follow its gate/up
// partial sums (at most 64 rows x 8 parts) in the partial buffer
constexpr int MU_ABUF_OFF = PBUF_OFF + 64 * 8 * 4;

// ---- expert-unit geometry (MK_OP_MOE_UNITS), shared by the runtime and the kernel -----------
// The down projection's row of I values is KS = parts(I) parts of Lp = I / KS values; lane l of a
// part holds values [8 l, 8 l + 8) for l < l8 = Lp / 8. Lane class q (0..7) is lanes q, q + 8,
// q + 16, q + 24: a level-2 subtree of the warp butterfly (xor 16, then xor 8).
__host__ __device__ constexpr int unit_parts(int I) { return I <= 256 ? 1 : I <= 512 ? 2 : I <= 1024 ? 4 : 8; }
// the lanes of class q that hold values
__host__ __device__ constexpr int unit_lanes(int q, int l8) { return l8 > q ? ((l8 - q + 7) / 8 < 4 ? (l8 - q + 7) / 8 : 4) : 0; }
// values before lane class q in a part of the regrouped down projection, per row
__host__ __device__ inline int unit_q_vals(int q, int l8) {
  int n = 0;
  for (int k = 0; k < q; ++k) n += unit_lanes(k, l8);
  return 8 * n;
}
// gate/up rows of row_bytes each per ring stage (a power of two dividing a lane's 16 rows)
__host__ __device__ constexpr int unit_w13_rows(int64_t row_bytes) {
  return STAGE_BYTES / row_bytes >= 16 ? 16 : STAGE_BYTES / row_bytes >= 8 ? 8 : STAGE_BYTES / row_bytes >= 4 ? 4
         : STAGE_BYTES / row_bytes >= 2 ? 2 : 1;
}
// regrouped down-projection rows of row_bytes each per ring stage: an even count, so a stage's
// bytes and its source offset stay multiples of 16 for FP8 rows of 8 nl bytes
__host__ __device__ constexpr int unit_w2_rows(int row_bytes) { return (STAGE_BYTES / row_bytes) & ~1; }
// the down projection's slot weights and slot outputs follow its activations (16-byte aligned)
__host__ __device__ constexpr int w2_aux_off(int ns, int inter) { return (ns * inter * 2 + 15) / 16 * 16; }
__host__ __device__ constexpr int w2_aux_bytes(int ns, int rows) { return (MAX_ROUTED + ns * rows) * 4; }

// ---- tables uploaded by the host ----------------------------------------------------------

struct __align__(16) OpDev {
  MkOp op;
  int32_t ntasks;
  int32_t task0;           // index of the operator's first task in the task table
  int32_t rps;             // rows per stage of its weight stream
  int32_t ksplit;          // warps sharing one row (GEMV K-split), else 1
  int32_t aux[4];          // producer-side dependency: aux[0] operator, aux[1] generations back
  int32_t dep_op[2];       // consumer-side dependencies: operators whose tasks must all be done
  int32_t dep_n[2];        // (-1: none), their task counts, and how many generations back
  int32_t dep_lag[2];
  int32_t pad[2];
};
static_assert(sizeof(OpDev) % 16 == 0, "OpDev is copied to shared memory in 16-byte pieces");

struct TaskDev {
  int32_t op;              // operator index
  int32_t idx;             // task index within the operator
  int32_t a, b;            // operator-specific range (rows, pairs, head group / split)
};

// one entry of a CTA's task list, in execution order
struct __align__(16) CtaTask {
  TaskDev t;
  int32_t next_op;         // operator of the CTA's next task (its first one after the last)
  int32_t signal;          // completions to add to the operator's event after this task: the
                           // length of the run of its tasks that this task ends, else 0
  int32_t pad[2];
};
static_assert(sizeof(CtaTask) == 32, "CtaTask is copied to shared memory in two 16-byte pieces");

struct DevStatus {
  uint32_t error, err_op, err_task, err_cta, err_info, aborted_ctas, abort_flag;
  uint32_t undrained;   // weight-stream stages a leaving producer could not drain in time
};

struct KernelParams {
  const OpDev* ops;
  const uint32_t* cta_off;       // [num_ctas + 1]
  const CtaTask* ctask;          // the CTAs' task lists, CTA c at [cta_off[c], cta_off[c + 1])
  uint32_t* events;              // [nops] completion counters (monotonic across iterations)
  uint32_t* arrive;              // [nops] arrival counters of the last-arriver finalizers
  DevStatus* status;
  float* amax_val;               // [max tasks] argmax partials
  int32_t* amax_idx;
  MkTraceRecord* trace;
  uint32_t* trace_count;
  uint32_t trace_cap;
  int32_t nops;
  int32_t iters;
  int32_t step;                  // iteration i runs at position step + 1 + i
  uint32_t gen0;                 // generation (1-based, global) of iteration 0
  int32_t block_op;              // debug: this operator's wait never succeeds (-1: none)
  int64_t timeout_ns;
  int32_t* meta_step;
  uint32_t ep_gen0;              // exchange tag of iteration 0 (expert parallelism; 1-based)
  const void* tmaps;             // tensor maps of the tensor-core attention operators (2 per operator)
  const uint16_t* units;         // the expert-unit operators' per-task unit lists (MuList)
};

// ---- shared memory ------------------------------------------------------------------------

enum { TR_READY = 0, TR_BODY = 1, TR_STAGES = 2, TR_WAIT = 3 };

struct __align__(128) Smem {
  uint8_t ring[NSTAGES][STAGE_BYTES];
  uint64_t full[NSTAGES];
  uint64_t empty[NSTAGES];
  __align__(16) uint8_t scratch[SCRATCH_BYTES];
  double red[NUM_CONSUMER_WARPS * 4];
  float wbest_v[NUM_CONSUMER_WARPS];
  int32_t wbest_i[NUM_CONSUMER_WARPS];
  int32_t bcast[8];
  uint32_t cta_abort;
  int32_t stage_aux[NSTAGES];   // a word the producer attaches to a stage (written before the stage's
                                // arrive, so the consumer that acquired the stage sees it)
  uint64_t tr[4];           // trace stamps of the running task (TR_*), thread 0
  KernelParams kp;          // the launch parameters
  __align__(16) OpDev od_buf[2];     // the running task's operator and the next one's (copied ahead)
  __align__(16) CtaTask ct_buf[2];
};

// ---- PTX wrappers -------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// global -> shared bulk copy (no tensor map); completes `bytes` of transaction on `bar`.
// Requirements: 16-byte aligned addresses, bytes a multiple of 16. The copy carries an L2
// evict-first policy: weights stream through L2 once per token, and without the hint they push
// the kernel's instructions, activations and split-KV partials out of L2.
__device__ __forceinline__ void bulk_g2s(void* sdst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(sdst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// global -> shared tiled tensor copy (TMA) of the 2-D box at element coordinates (x, y) of the
// tensor map `tmap` (a CUtensorMap in global memory); completes its bytes on `bar`. x times the
// element size must be a multiple of 16 bytes; the destination is 1024-byte aligned for the
// 128-byte swizzle. Never a multicast form: the source may be any GPU's memory.
__device__ __forceinline__ void tma_load_2d(void* sdst, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(sdst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// generic-proxy writes to shared memory made visible to later async-proxy (TMA) accesses
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// tensor-core fragments: four 8x8 BF16 matrices from shared memory (thread t gives the address of
// row t % 8 of matrix t / 8); .trans transposes each matrix
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
// D = A B + D on the tensor cores: A 16x16 (row-major fragment), B 16x8 (column-major), BF16
// inputs, FP32 accumulators
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// explicit shared-memory loads (the address is a shared-window offset, smem_u32)
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint16_t lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float ldsf(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
// 16-byte global -> shared copy that bypasses registers (completed by cp_async_wait_all)
__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// expert-parallel exchange words: one 64-bit access (single-copy atomic for an aligned 64-bit
// scalar), relaxed at system scope (another GPU's memory, or this GPU's memory that another GPU
// writes)
// a value with its iteration tag as one 64-bit word (single-copy atomic): a reader that sees the
// tag it expects also sees the value, with no fence and no counter
__device__ __forceinline__ void st_relaxed_gpu_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_gpu_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acqrel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// loads of activations written by other CTAs in this launch: L2 only (never a stale L1 line)
__device__ __forceinline__ uint4 ldcg16(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint32_t ldcg_u16(const uint16_t* p) { return (uint32_t)__ldcg(p); }
__device__ __forceinline__ float ldcg_f32(const float* p) { return __ldcg(p); }

}  // namespace mk
