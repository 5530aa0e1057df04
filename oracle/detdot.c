/* detdot.c -- C restatement of the CPU oracle's two heaviest loops (oracle/detmath.py dot_rows
 * and oracle/numpy_ref.py mla_attend), operation for operation, so that a full 27-layer greedy
 * decode can be checked on the host in about a second per token.
 *
 * TEST INFRASTRUCTURE. Loaded only by oracle/detmath.py (ctypes); only tests/, the smoke check and
 * bench.py's CPU-baseline legs reach it. The numpy functions stay the specification: the C results
 * must equal theirs bit for bit (tests/test_oracle_detmath.py), and detmath.py uses numpy when this
 * library has not been built.
 *
 * Arithmetic: IEEE binary32 with round to nearest even, no contraction (built with
 * -ffp-contract=off, never -ffast-math; threads are plain pthreads). Every product of two BF16 values is exact in binary32.
 *   row dot (detmath.dot_rows): the row is KS equal parts of kp values; in a part, lane l (of 32)
 *     takes the 8-value vectors v = l + 32 j (j < maxv, v * 8 < kp) and adds their products in the
 *     order (j, t = 0..7) into a0 (t even) and a1 (t odd); the lane value is a0 + a1; lane 0 of the
 *     xor butterfly (offsets 16, 8, 4, 2, 1) is the part's sum; parts are added in order.
 *   attention (numpy_ref.mla_attend): per split and head, scores by lanes (contiguous latent then
 *     rope columns per lane, then the butterfly) times the scale; m = max; p = det_exp(s - m);
 *     l = lane sum of p; o = (sequential sum over rows of bf16(p) c_kv) / l; lse = m + det_log(l).
 * det_exp / det_log are detmath.py's Cody-Waite + Taylor and atanh-series routines; their FP32
 * constants come from Python (od_set_consts) so both sides use the same bits.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---- a static-schedule parallel for over [0, n) on pthreads (ORACLE_THREADS, else every core) */
typedef void (*od_body_fn)(void* ctx, int64_t lo, int64_t hi);
typedef struct { od_body_fn fn; void* ctx; int64_t lo, hi; } od_chunk;

static void* od_run_chunk(void* p) {
  od_chunk* c = (od_chunk*)p;
  c->fn(c->ctx, c->lo, c->hi);
  return NULL;
}

static int od_threads(void) {
  const char* e = getenv("ORACLE_THREADS");
  long n = e ? strtol(e, NULL, 10) : sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  if (n > 256) n = 256;
  return (int)n;
}

static void od_parallel_for(int64_t n, int64_t min_chunk, od_body_fn fn, void* ctx) {
  int t = od_threads();
  if ((int64_t)t * min_chunk > n) t = (int)(n / min_chunk);
  if (t <= 1) { fn(ctx, 0, n); return; }
  pthread_t th[256];
  od_chunk ch[256];
  int joined[256];
  for (int i = 0; i < t; ++i) {
    ch[i].fn = fn;
    ch[i].ctx = ctx;
    ch[i].lo = n * i / t;
    ch[i].hi = n * (i + 1) / t;
    joined[i] = 0;
  }
  for (int i = 1; i < t; ++i)     /* a chunk whose thread cannot start runs on this one */
    joined[i] = pthread_create(&th[i], NULL, od_run_chunk, &ch[i]) == 0;
  od_run_chunk(&ch[0]);
  for (int i = 1; i < t; ++i) {
    if (joined[i]) pthread_join(th[i], NULL);
    else od_run_chunk(&ch[i]);
  }
}

static float C_LOG2E, C_LN2_HI, C_LN2_LO, C_SQRT2, C_EXP_LO, C_EXP_HI;
static float C_EXP[8], C_LOG[5];

void od_set_consts(const float* c) {
  C_LOG2E = c[0]; C_LN2_HI = c[1]; C_LN2_LO = c[2]; C_SQRT2 = c[3]; C_EXP_LO = c[4]; C_EXP_HI = c[5];
  for (int i = 0; i < 8; ++i) C_EXP[i] = c[6 + i];
  for (int i = 0; i < 5; ++i) C_LOG[i] = c[14 + i];
}

static inline float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf_bits(uint16_t b) { return f_of((uint32_t)b << 16); }
static inline float bf16r(float x) {
  uint32_t u = u_of(x);
  const uint32_t lsb = (u >> 16) & 1u;
  u = (u + 0x7FFFu + lsb) & 0xFFFF0000u;
  return f_of(u);
}

/* lane 0 of the xor butterfly over a[32] (a is overwritten) */
static inline float butterfly32(float* a) {
  for (int half = 16; half > 0; half >>= 1)
    for (int l = 0; l < half; ++l) a[l] = a[l] + a[l + half];
  return a[0];
}

static void parts_of(int64_t K, int* ks, int64_t* kp, int* maxv) {
  int k = 8;
  if (K <= 2048) {
    for (k = 1; k < 8 && K > 256 * k; k *= 2) {}
  }
  *ks = k;
  *kp = K / k;
  *maxv = (int)((*kp + 255) / 256);
}

#define DOT_ROW_BODY(LOADW)                                                   \
  float d = 0.0f;                                                             \
  for (int p = 0; p < ks; ++p) {                                              \
    float lane[32];                                                           \
    for (int l = 0; l < 32; ++l) {                                            \
      float a0 = 0.0f, a1 = 0.0f;                                             \
      for (int j = 0; j < maxv; ++j) {                                        \
        const int64_t v = l + 32 * (int64_t)j;                                \
        if (v * 8 >= kp) break;                                               \
        const int64_t o = (int64_t)p * kp + v * 8;                            \
        a0 = a0 + LOADW(o + 0) * x[o + 0];                                    \
        a1 = a1 + LOADW(o + 1) * x[o + 1];                                    \
        a0 = a0 + LOADW(o + 2) * x[o + 2];                                    \
        a1 = a1 + LOADW(o + 3) * x[o + 3];                                    \
        a0 = a0 + LOADW(o + 4) * x[o + 4];                                    \
        a1 = a1 + LOADW(o + 5) * x[o + 5];                                    \
        a0 = a0 + LOADW(o + 6) * x[o + 6];                                    \
        a1 = a1 + LOADW(o + 7) * x[o + 7];                                    \
      }                                                                       \
      lane[l] = a0 + a1;                                                      \
    }                                                                         \
    const float part = butterfly32(lane);                                     \
    d = p == 0 ? part : d + part;                                             \
  }

typedef struct { const void* W; int64_t K; const float* x; float* out; int ks, maxv; int64_t kp; } od_dot_ctx;

static void od_dot_bf16_body(void* vc, int64_t lo, int64_t hi) {
  const od_dot_ctx* c = (const od_dot_ctx*)vc;
  const int ks = c->ks, maxv = c->maxv;
  const int64_t kp = c->kp;
  const float* x = c->x;
  for (int64_t n = lo; n < hi; ++n) {
    const uint16_t* w = (const uint16_t*)c->W + n * c->K;
#define LW(i) bf_bits(w[i])
    DOT_ROW_BODY(LW)
#undef LW
    c->out[n] = d;
  }
}

static void od_dot_f32_body(void* vc, int64_t lo, int64_t hi) {
  const od_dot_ctx* c = (const od_dot_ctx*)vc;
  const int ks = c->ks, maxv = c->maxv;
  const int64_t kp = c->kp;
  const float* x = c->x;
  for (int64_t n = lo; n < hi; ++n) {
    const float* w = (const float*)c->W + n * c->K;
#define LW(i) w[i]
    DOT_ROW_BODY(LW)
#undef LW
    c->out[n] = d;
  }
}

/* out[n] = dot of row n of W [N, K] (BF16 bit patterns) with x [K] (FP32 holding BF16 values) */
void od_dot_rows_bf16(const uint16_t* W, int64_t N, int64_t K, const float* x, float* out) {
  od_dot_ctx c = {W, K, x, out, 0, 0, 0};
  parts_of(K, &c.ks, &c.kp, &c.maxv);
  od_parallel_for(N, 1 + (1 << 16) / (K > 0 ? K : 1), od_dot_bf16_body, &c);
}

/* the same with W as FP32 values (each a BF16 value) */
void od_dot_rows_f32(const float* W, int64_t N, int64_t K, const float* x, float* out) {
  od_dot_ctx c = {W, K, x, out, 0, 0, 0};
  parts_of(K, &c.ks, &c.kp, &c.maxv);
  od_parallel_for(N, 1 + (1 << 16) / (K > 0 ? K : 1), od_dot_f32_body, &c);
}

float od_det_exp(float x) {
  if (isnan(x)) return NAN;
  if (x < C_EXP_LO) return 0.0f;
  if (x > C_EXP_HI) return INFINITY;
  const float k = rintf(x * C_LOG2E);
  const float r = (x - k * C_LN2_HI) - k * C_LN2_LO;
  float p = C_EXP[7];
  for (int n = 6; n >= 0; --n) p = p * r + C_EXP[n];
  const float scale = f_of((uint32_t)((int32_t)k + 127) << 23);
  return p * scale;
}

float od_det_log(float x) {
  if (isnan(x) || x < 0.0f) return NAN;
  if (x == 0.0f) return -INFINITY;
  if (isinf(x)) return INFINITY;
  int esub = 0;
  float xs = x;
  if (x < f_of(0x00800000u)) { xs = x * 16777216.0f; esub = 24; }
  const uint32_t bits = u_of(xs);
  int32_t e = (int32_t)(bits >> 23) - 127 - esub;
  float m = f_of((bits & 0x7FFFFFu) | 0x3F800000u);
  if (m > C_SQRT2) { m = m * 0.5f; e += 1; }
  const float t = (m - 1.0f) / (m + 1.0f);
  const float t2 = t * t;
  float s = C_LOG[4];
  s = s * t2 + C_LOG[3];
  s = s * t2 + C_LOG[2];
  s = s * t2 + C_LOG[1];
  s = s * t2 + C_LOG[0];
  const float logm = (t + t) * s;
  const float ef = (float)e;
  return ef * C_LN2_HI + (ef * C_LN2_LO + logm);
}

typedef struct {
  const float *ql_nope, *q_pe, *c_kv, *k_pe;
  int nh, dc, dr, step, split;
  float scale;
  float* partials;
} od_att_ctx;

/* one (split, head) pair per unit: u = j * nh + h */
static void od_attend_body(void* vc, int64_t lo_u, int64_t hi_u) {
  const od_att_ctx* c = (const od_att_ctx*)vc;
  const int nh = c->nh, dc = c->dc, dr = c->dr, row = dc + 1;
  const int lc = dc >= 32 ? dc / 32 : 1, rp = dr >= 32 ? dr / 32 : 1;
  float s[4096], pb[4096];
  for (int64_t u = lo_u; u < hi_u; ++u) {
    const int j = (int)(u / nh), h = (int)(u % nh);
    const int lo = j * c->split;
    float* out = c->partials + ((size_t)j * nh + h) * row;
    if (lo > c->step) { out[dc] = -INFINITY; continue; }
    const int hi = lo + c->split < c->step + 1 ? lo + c->split : c->step + 1;
    const int rows = hi - lo;
    const float* q = c->ql_nope + (size_t)h * dc;
    const float* qr = c->q_pe + (size_t)h * dr;
    float mx = -INFINITY;
    for (int r = 0; r < rows; ++r) {
      const float* cr = c->c_kv + (size_t)(lo + r) * dc;
      const float* kr = c->k_pe + (size_t)(lo + r) * dr;
      float acc[32];
      for (int l = 0; l < 32; ++l) {
        float a = 0.0f;
        for (int m = 0; m < lc; ++m) {
          const int col = l * lc + m;
          if (col < dc) a = a + cr[col] * q[col];
        }
        for (int m = 0; m < rp; ++m) {
          const int col = l * rp + m;
          if (col < dr) a = a + kr[col] * qr[col];
        }
        acc[l] = a;
      }
      s[r] = butterfly32(acc) * c->scale;
      if (s[r] > mx) mx = s[r];
    }
    float lanes[32];
    for (int l = 0; l < 32; ++l) lanes[l] = 0.0f;
    for (int r = 0; r < rows; ++r) {
      const float p = od_det_exp(s[r] - mx);
      lanes[r % 32] = lanes[r % 32] + p;
      pb[r] = bf16r(p);
    }
    const float l_sum = butterfly32(lanes);
    for (int col = 0; col < dc; ++col) {
      float a = 0.0f;
      for (int r = 0; r < rows; ++r) a = a + pb[r] * c->c_kv[(size_t)(lo + r) * dc + col];
      out[col] = a / l_sum;
    }
    out[dc] = mx + od_det_log(l_sum);
  }
}

/* numpy_ref.mla_attend: partials [n_splits, nh, dc + 1] (o, then lse at column dc) over cache rows
   [0, step]; splits of `split` rows (at most 4096); empty splits get o = 0 and lse = -inf */
void od_mla_attend(const float* ql_nope, const float* q_pe, const float* c_kv, const float* k_pe, int nh, int dc,
                   int dr, int step, float scale, int split, int n_splits, float* partials) {
  memset(partials, 0, sizeof(float) * (size_t)n_splits * nh * (dc + 1));
  od_att_ctx c = {ql_nope, q_pe, c_kv, k_pe, nh, dc, dr, step, split, scale, partials};
  od_parallel_for((int64_t)n_splits * nh, 1, od_attend_body, &c);
}
