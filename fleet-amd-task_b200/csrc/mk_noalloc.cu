// mk_noalloc.cu -- the MLA decode attention (split-KV partials, then the merge and the W_uv
// product) as ONE entry point that allocates no device memory: mk_mla_decode_noalloc.
//
// Who needs it: a caller that cannot call cudaMalloc at this point of its program. Typical cases
// are engines that reserve all of HBM for their own pool before serving (a stray cudaMalloc fails
// or fragments that pool), code that runs while the caller's allocator holds its own lock, and
// latency-critical loops where the implicit synchronisation of cudaMalloc/cudaFree would stall the
// pipeline. The persistent kernel's handle (mk_finalize) allocates its tables and counters once;
// this entry point needs no handle at all.
//
// Where the scratch lives: the split-KV partials (the only intermediate this computation needs)
// are a file-scope __device__ array of MLA_NOALLOC_MAX_FLOATS floats (2 MiB), which every GPU
// that loads the library keeps until the process exits. Host code cannot pass the array's name to
// a kernel (on the host it names a stand-in, not a device address), so the first call on each
// device looks the device address up with cudaGetSymbolAddress while that device is current, and
// later calls reuse it. That first call should therefore happen before any stream capture.
//
// Sharing: every call on a device uses the same array, which keeps the last call's values. Calls
// that overlap on the GPU (two streams, or two host threads) race on it and must be ordered by the
// caller. Nothing has to start at zero: each call writes every partial row that it then reads.
//
// Arithmetic: identical to the persistent kernel's MK_OP_MLA_ATTEND + MK_OP_MLA_MERGE_UV (FP32 sums in
// the same specified orders, det_exp / det_log), so the two agree bit for bit.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/fleet_mk.h"
#include "detmath.cuh"

namespace mk {
int set_last_error(int code, const char* msg);   // mk_runtime.cu: the message mk_last_error() returns
}

using namespace mk;

namespace {

constexpr int NA_MAX_SPLITS = 64;
constexpr int NA_MAX_HEADS = 16;
constexpr int NA_MAX_DC = 512;
constexpr int NA_PROW = ((NA_MAX_DC + 1 + 3) / 4) * 4;
constexpr int NA_THREADS = 256;
constexpr int NA_MAX_SPLIT_ROWS = 256;
constexpr int MLA_NOALLOC_MAX_FLOATS = NA_MAX_SPLITS * NA_MAX_HEADS * NA_PROW;   // 528,384 floats

static __device__ __align__(256) float g_mla_partials[MLA_NOALLOC_MAX_FLOATS];

constexpr int NA_MAX_DEVICES = 64;
std::mutex g_mu;
float* g_dev_ptr[NA_MAX_DEVICES] = {};

struct NaArgs {
  const uint16_t* ql_nope;   // [nh, d_c]
  const uint16_t* q_pe;      // [nh, d_r]
  const uint16_t* c_kv;      // [s_max, d_c]
  const uint16_t* k_pe;      // [s_max, d_r]
  const uint16_t* w_uv;      // [nh, d_v, d_c]
  uint16_t* attn;            // [nh * d_v]
  float* partials;           // the static array's device address
  int nh, d_c, d_r, d_v, pos, split, live, prow;
  float scale;
};

// one block per (head, live split): the split's scores, softmax statistics and P.V, in the same
// FP32 orders as the persistent kernel's attend task
__global__ void __launch_bounds__(NA_THREADS) na_attend_kernel(NaArgs a) {
  __shared__ float sc[NA_MAX_SPLIT_ROWS];
  __shared__ float pb[NA_MAX_SPLIT_ROWS];
  __shared__ float stat[2];
  const int h = blockIdx.x, j = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lo = j * a.split, hi = min(lo + a.split, a.pos + 1);
  const int rows = hi - lo;
  // lane l owns the contiguous latent columns [l * lc, l * lc + lc) and rope columns
  // [l * rp, l * rp + rp) (one rope column for lanes l < d_r when d_r < 32)
  const int lc = a.d_c / 32, rp = a.d_r >= 32 ? a.d_r / 32 : 1;
  float qn[NA_MAX_DC / 32], qp[2];
#pragma unroll
  for (int m = 0; m < NA_MAX_DC / 32; ++m)
    qn[m] = m < lc ? bf16_bits_to_f32(a.ql_nope[(size_t)h * a.d_c + lane * lc + m]) : 0.0f;
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const int col = lane * rp + m;
    qp[m] = (m < rp && col < a.d_r) ? bf16_bits_to_f32(a.q_pe[(size_t)h * a.d_r + col]) : 0.0f;
  }
  for (int r = warp; r < rows; r += NA_THREADS / 32) {
    const uint16_t* crow = a.c_kv + (size_t)(lo + r) * a.d_c + lane * lc;
    const uint16_t* krow = a.k_pe + (size_t)(lo + r) * a.d_r + lane * rp;
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < NA_MAX_DC / 32; ++m)
      if (m < lc) acc = fmaf(bf16_bits_to_f32(crow[m]), qn[m], acc);
#pragma unroll
    for (int m = 0; m < 2; ++m)
      if (m < rp && lane * rp + m < a.d_r) acc = fmaf(bf16_bits_to_f32(krow[m]), qp[m], acc);
    acc = warp_butterfly(acc);
    if (lane == 0) sc[r] = __fmul_rn(acc, a.scale);
  }
  __syncthreads();
  if (warp == 0) {
    float mx = -__int_as_float(0x7F800000);
    for (int r = lane; r < rows; r += 32) mx = fmaxf(mx, sc[r]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int r = lane; r < rows; r += 32) {
      const float p = det_exp(__fsub_rn(sc[r], mx));
      pb[r] = round_bf16(p);
      sum = __fadd_rn(sum, p);
    }
    sum = warp_butterfly(sum);
    if (lane == 0) { stat[0] = mx; stat[1] = sum; }
  }
  __syncthreads();
  float* out = a.partials + ((size_t)j * a.nh + h) * a.prow;
  for (int c = threadIdx.x; c < a.d_c; c += NA_THREADS) {
    float acc = 0.0f;
    for (int r = 0; r < rows; ++r) acc = fmaf(bf16_bits_to_f32(a.c_kv[(size_t)(lo + r) * a.d_c + c]), pb[r], acc);
    out[c] = __fdiv_rn(acc, stat[1]);
  }
  if (threadIdx.x == 0) out[a.d_c] = __fadd_rn(stat[0], det_log(stat[1]));
}

// one block per head: merge the live splits into o (BF16), then attn[h, v] = W_uv[h, v] . o as
// the persistent kernel's row dot: the row is KS equal parts of at most 256 values (KS 1 for
// d_c <= 256, else 2); in each part lane l takes the part's 8-value vector l, adds the even
// products into a0 and the odd ones into a1, then a0 + a1 and the butterfly gives the part's sum;
// the part sums are added in part order
__global__ void __launch_bounds__(NA_THREADS) na_merge_kernel(NaArgs a) {
  __shared__ __align__(16) uint16_t ob[NA_MAX_DC];
  const int h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < a.d_c; c += NA_THREADS) {
    float M = -__int_as_float(0x7F800000);
    for (int j = 0; j < a.live; ++j) M = fmaxf(M, a.partials[((size_t)j * a.nh + h) * a.prow + a.d_c]);
    float num = 0.0f, den = 0.0f;
    for (int j = 0; j < a.live; ++j) {
      const float* row = a.partials + ((size_t)j * a.nh + h) * a.prow;
      const float w = det_exp(__fsub_rn(row[a.d_c], M));
      num = __fadd_rn(num, __fmul_rn(w, row[c]));
      den = __fadd_rn(den, w);
    }
    ob[c] = (uint16_t)f32_to_bf16_bits(__fdiv_rn(num, den));
  }
  __syncthreads();
  const int ks = a.d_c <= 256 ? 1 : 2, lp = a.d_c / ks;
  for (int v = warp; v < a.d_v; v += NA_THREADS / 32) {
    const uint16_t* wrow = a.w_uv + ((size_t)h * a.d_v + v) * a.d_c;
    float d = 0.0f;
    for (int p = 0; p < ks; ++p) {
      float a0 = 0.0f, a1 = 0.0f;
      if (lane * 8 < lp) {
        const int base = p * lp + lane * 8;
        for (int t = 0; t < 8; ++t) {
          const float w = bf16_bits_to_f32(wrow[base + t]);
          const float x = bf16_bits_to_f32((uint32_t)ob[base + t]);
          if (t % 2 == 0) a0 = fmaf(w, x, a0);
          else a1 = fmaf(w, x, a1);
        }
      }
      const float part = warp_butterfly(__fadd_rn(a0, a1));
      d = p == 0 ? part : __fadd_rn(d, part);
    }
    if (lane == 0) a.attn[(size_t)h * a.d_v + v] = (uint16_t)f32_to_bf16_bits(d);
  }
}

int na_fail(int code, const char* msg) { return mk::set_last_error(code, msg); }

}  // namespace

extern "C" int mk_mla_decode_noalloc(const void* ql_nope, const void* q_pe, const void* c_kv, const void* k_pe,
                                     const void* w_uv, void* attn_out, int32_t nh, int32_t d_c, int32_t d_r,
                                     int32_t d_v, int32_t pos, int32_t split, float softmax_scale, void* stream) {
  if (!ql_nope || !q_pe || !c_kv || !k_pe || !w_uv || !attn_out) return na_fail(MK_EINVAL, "null pointer");
  if (nh < 1 || nh > NA_MAX_HEADS || d_c < 32 || d_c > NA_MAX_DC || d_c % 32 || d_r < 2 || (d_r > 32 && d_r != 64) || d_r % 2 ||
      d_v < 1 || split < 1 || split > NA_MAX_SPLIT_ROWS || pos < 0)
    return na_fail(MK_EINVAL, "shape outside the entry point's limits (heads <= 16, d_c <= 512, d_r <= 32 or 64, "
                              "split <= 256)");
  const int live = (pos + 1 + split - 1) / split;
  const int prow = ((d_c + 1 + 3) / 4) * 4;
  if (live > NA_MAX_SPLITS || (int64_t)live * nh * prow > MLA_NOALLOC_MAX_FLOATS)
    return na_fail(MK_EINVAL, "pos + 1 needs more than 64 splits: the static scratch holds 64 x 16 x 516 floats");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= NA_MAX_DEVICES)
    return na_fail(MK_ECUDA, "cudaGetDevice failed or device ordinal out of range");
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_dev_ptr[dev]) {
      // set-up, once per device, with that device current: the array's device address
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_mla_partials);
      if (e != cudaSuccess) return na_fail(MK_ECUDA, cudaGetErrorString(e));
      g_dev_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_dev_ptr[dev];
  }
  NaArgs a;
  a.ql_nope = static_cast<const uint16_t*>(ql_nope);
  a.q_pe = static_cast<const uint16_t*>(q_pe);
  a.c_kv = static_cast<const uint16_t*>(c_kv);
  a.k_pe = static_cast<const uint16_t*>(k_pe);
  a.w_uv = static_cast<const uint16_t*>(w_uv);
  a.attn = static_cast<uint16_t*>(attn_out);
  a.partials = scratch;
  a.nh = nh; a.d_c = d_c; a.d_r = d_r; a.d_v = d_v; a.pos = pos; a.split = split; a.live = live; a.prow = prow;
  a.scale = softmax_scale;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  na_attend_kernel<<<dim3((unsigned)nh, (unsigned)live), NA_THREADS, 0, s>>>(a);
  na_merge_kernel<<<dim3((unsigned)nh), NA_THREADS, 0, s>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return na_fail(MK_ECUDA, cudaGetErrorString(e));
  return MK_OK;
}
