/*
 * q3_oracle.c -- CPU restatement of the Qwen3-0.6B Q8_0 decode hot path of
 * abourramouss/qwen3-iree (model/qwen3_full.mlir, kernels/cuda and kernels/mlir,
 * tools/create_q8_irpa.py).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke test
 * and bench.py's CPU-baseline legs load it; the CUDA library never does.
 *
 * Pinning:
 *   - quantize / dequant: against golden vectors produced by the reference's
 *     own tools/create_q8_irpa.py functions (tests/golden/make_golden.py);
 *   - q3o_gemv_q8_cuda / q3o_gemv_f16: bit-for-bit against the reference's
 *     kernels/cuda/dispatch_{3,4,12,18,20,24}.cu compiled for sm_100a and run
 *     on a B200 (oracle/Makefile builds them into oracle/_ref/);
 *   - norms, RoPE, attention, SwiGLU, argmax and the layer order follow
 *     model/qwen3_full.mlir as read; IREE (not vendored, unpinned version)
 *     chooses their reduction order on the GPU, so for those ops the order is
 *     fixed here and stated beside each function ("parity unpinned" for the
 *     order, exact for the formula).
 *
 * Floating point rules: compile without -ffast-math and with
 * -ffp-contract=off; every fused multiply-add is an explicit fmaf().  f16
 * values are IEEE binary16 bit patterns; conversions round to nearest even.
 */
#include "q3_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---------------------------------------------------------------------- */
/* A small persistent thread pool (this image's gcc has no OpenMP runtime). */
/* pool_for(n, fn, ctx) runs fn(ctx, begin, end) over static slices of     */
/* [0, n); results never depend on the thread count (rows are independent). */
/* ---------------------------------------------------------------------- */
typedef void (*task_fn)(void* ctx, int64_t begin, int64_t end);
#define POOL_MAX 256
static struct {
  pthread_mutex_t mu;
  pthread_cond_t cv_go, cv_done;
  pthread_t th[POOL_MAX];
  int nthreads, started, pending;
  int64_t gen, total;
  task_fn fn;
  void* ctx;
} g_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER};
static int g_want_threads = 0;

static void slice(int64_t total, int n, int t, int64_t* b, int64_t* e) {
  *b = total * t / n;
  *e = total * (t + 1) / n;
}

static void* pool_worker(void* arg) {
  const int t = (int)(intptr_t)arg;
  int64_t seen = 0;
  for (;;) {
    pthread_mutex_lock(&g_pool.mu);
    while (g_pool.gen == seen) pthread_cond_wait(&g_pool.cv_go, &g_pool.mu);
    seen = g_pool.gen;
    task_fn fn = g_pool.fn;
    void* ctx = g_pool.ctx;
    const int64_t total = g_pool.total;
    const int n = g_pool.nthreads;
    pthread_mutex_unlock(&g_pool.mu);
    int64_t b, e;
    slice(total, n, t, &b, &e);
    if (b < e) fn(ctx, b, e);
    pthread_mutex_lock(&g_pool.mu);
    if (--g_pool.pending == 0) pthread_cond_signal(&g_pool.cv_done);
    pthread_mutex_unlock(&g_pool.mu);
  }
  return NULL;
}

static void pool_start(void) {
  if (g_pool.started) return;
  int n = g_want_threads > 0 ? g_want_threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  if (n > POOL_MAX) n = POOL_MAX;
  g_pool.nthreads = n;
  for (int t = 1; t < n; ++t) pthread_create(&g_pool.th[t], NULL, pool_worker, (void*)(intptr_t)t);
  g_pool.started = 1;
}

/* One pool_for at a time: the pool has a single task slot, and callers may
 * come from several host threads (the weight generator quantises layers from
 * a thread pool). */
static pthread_mutex_t g_pool_call_mu = PTHREAD_MUTEX_INITIALIZER;

static void pool_for_locked(int64_t total, task_fn fn, void* ctx);

static void pool_for(int64_t total, task_fn fn, void* ctx) {
  pthread_mutex_lock(&g_pool_call_mu);
  pool_for_locked(total, fn, ctx);
  pthread_mutex_unlock(&g_pool_call_mu);
}

static void pool_for_locked(int64_t total, task_fn fn, void* ctx) {
  pool_start();
  const int n = g_pool.nthreads;
  if (n == 1 || total < 2) {
    fn(ctx, 0, total);
    return;
  }
  pthread_mutex_lock(&g_pool.mu);
  g_pool.fn = fn;
  g_pool.ctx = ctx;
  g_pool.total = total;
  g_pool.pending = n - 1;
  g_pool.gen++;
  pthread_cond_broadcast(&g_pool.cv_go);
  pthread_mutex_unlock(&g_pool.mu);
  int64_t b, e;
  slice(total, n, 0, &b, &e);
  if (b < e) fn(ctx, b, e);
  pthread_mutex_lock(&g_pool.mu);
  while (g_pool.pending > 0) pthread_cond_wait(&g_pool.cv_done, &g_pool.mu);
  pthread_mutex_unlock(&g_pool.mu);
}

/* RMS epsilon: f32 of 1e-6 (model/qwen3_full.mlir:61-64, :607) */
static const float kEps = 9.99999997e-7f;
/* attention scale rsqrt(128) (model/qwen3_full.mlir:722-723), correctly rounded */
static const float kAttnScale = 0.0883883476483184405f;

float q3o_h2f(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

uint16_t q3o_f2h(float f) {
  _Float16 v = (_Float16)f;
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

/* exp(x) in f32 by Cody-Waite range reduction (x = n*ln2 + r, |r| <= ln2/2)
 * and the degree-7 Taylor polynomial of e^r in Horner form, then an exact
 * scaling by 2^n.  The CUDA kernels run the identical operation sequence, so
 * both sides produce the same bits.  Error is within 2 ulp of exp (tested). */
float q3o_expf(float x) {
  if (x != x) return x;
  if (x > 89.0f) return INFINITY;
  if (x < -104.0f) return 0.0f;
  const float n = rintf(x * 1.44269504088896341f);
  float r = fmaf(n, -0.693145751953125f, x);    /* ln2 high part, 16 bits */
  r = fmaf(n, -1.428606820309417e-6f, r);       /* ln2 - high part */
  float p = 1.984126984126984e-4f;              /* 1/7! */
  p = fmaf(p, r, 1.388888888888889e-3f);        /* 1/6! */
  p = fmaf(p, r, 8.333333333333333e-3f);        /* 1/5! */
  p = fmaf(p, r, 4.166666666666667e-2f);        /* 1/4! */
  p = fmaf(p, r, 1.666666666666667e-1f);        /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int k = (int)n;
  union { uint32_t u; float f; } s;
  if (k > 127) {
    p = p * 2.0f;
    k -= 1;
  }
  if (k < -126) {
    s.u = (uint32_t)(k + 64 + 127) << 23;
    p = p * s.f;
    s.u = (uint32_t)(-64 + 127) << 23;
    return p * s.f;
  }
  s.u = (uint32_t)(k + 127) << 23;
  return p * s.f;
}

/* ---------------------------------------------------------------------- */
/* Q8_0 format                                                            */
/* ---------------------------------------------------------------------- */

/* tools/create_q8_irpa.py:103-118 (quantize_q8_0): per block of 32,
 * scale = amax/127 in f32 (0 -> 1.0), q = round-half-even(w/scale) clipped to
 * [-128,127], scale stored as f16 little-endian ahead of the 32 int8. */
typedef struct {
  const float* w;
  uint8_t* out;
} quant_ctx;

static void quant_task(void* vctx, int64_t b0, int64_t b1) {
  const quant_ctx* c = (const quant_ctx*)vctx;
  const float* w = c->w;
  uint8_t* out = c->out;
  for (int64_t b = b0; b < b1; ++b) {
    const float* blk = w + b * Q3O_QBLK;
    float amax = 0.0f;
    for (int j = 0; j < Q3O_QBLK; ++j) {
      const float a = fabsf(blk[j]);
      if (a > amax) amax = a;
    }
    float scale = amax / 127.0f;
    if (scale == 0.0f) scale = 1.0f;
    const uint16_t sh = q3o_f2h(scale);
    uint8_t* o = out + b * Q3O_QBYTES;
    o[0] = (uint8_t)(sh & 0xff);
    o[1] = (uint8_t)(sh >> 8);
    for (int j = 0; j < Q3O_QBLK; ++j) {
      float q = rintf(blk[j] / scale);
      if (q < -128.0f) q = -128.0f;
      if (q > 127.0f) q = 127.0f;
      o[2 + j] = (uint8_t)(int8_t)q;
    }
  }
}

void q3o_quantize_q8_0(const float* w, int64_t n, uint8_t* out) {
  quant_ctx c = {w, out};
  pool_for(n / Q3O_QBLK, quant_task, &c);
}

/* tools/create_q8_irpa.py:121-129 (dequant_q8_0): f32(scale_f16) * f32(q),
 * exact in f32 (11-bit by 8-bit product). */
typedef struct {
  const uint8_t* raw;
  float* out;
} deq_ctx;

static void deq_task(void* vctx, int64_t b0, int64_t b1) {
  const deq_ctx* c = (const deq_ctx*)vctx;
  for (int64_t b = b0; b < b1; ++b) {
    const uint8_t* blk = c->raw + b * Q3O_QBYTES;
    const float s = q3o_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
    for (int j = 0; j < Q3O_QBLK; ++j) c->out[b * Q3O_QBLK + j] = s * (float)(int8_t)blk[2 + j];
  }
}

void q3o_dequant_q8_0(const uint8_t* raw, int64_t n, float* out) {
  deq_ctx c = {raw, out};
  pool_for(n / Q3O_QBLK, deq_task, &c);
}

/* ---------------------------------------------------------------------- */
/* GEMVs                                                                  */
/* ---------------------------------------------------------------------- */

/* The warp butterfly of the reference kernels: five __shfl_xor_sync steps
 * with offsets 16,8,4,2,1 (kernels/cuda/dispatch_3.cu:45-46,
 * kernels/mlir/dispatch_12_gpu.mlir:132-141); every lane ends with the same
 * value because a+b == b+a. */
static float butterfly_sum(const float* v32) {
  float v[32], t[32];
  memcpy(v, v32, sizeof(v));
  for (int off = 16; off > 0; off >>= 1) {
    for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ off];
    memcpy(v, t, sizeof(v));
  }
  return v[0];
}

static void x_to_f32(const uint16_t* x, float* xf, int K) {
  for (int k = 0; k < K; ++k) xf[k] = q3o_h2f(x[k]);
}

/* Q8_0 GEMV in the order of the reference's GPU-dialect kernels
 * (kernels/mlir/dispatch_12_gpu.mlir:100-129, identical in dispatch_3/4/18/20):
 * lane l walks blocks b = l, l+32, ...; per block inner = sum_j q_j*x_j as an
 * f32 fma chain over j = 0..31, then acc = fma(scale, inner, acc); the lane
 * partials meet in the butterfly and the result is rounded to f16. */
typedef struct {
  const uint8_t* w;
  const float* xf;
  const float* xT;
  uint16_t* y;
  int nb, ngroups;
} gemv_ctx;

static void gemv_q8_mlir_task(void* vctx, int64_t n0, int64_t n1) {
  const gemv_ctx* c = (const gemv_ctx*)vctx;
  const int nb = c->nb, ngroups = c->ngroups;
  const int64_t rowbytes = (int64_t)nb * Q3O_QBYTES;
  float qT[32 * 32];
  float inner[32], sc[32];
  for (int64_t n = n0; n < n1; ++n) {
    const uint8_t* row = c->w + n * rowbytes;
    float acc[32] = {0};
    for (int g = 0; g < ngroups; ++g) {
      const int lanes = (nb - g * 32) < 32 ? (nb - g * 32) : 32;
      for (int l = 0; l < 32; ++l) {
        if (l < lanes) {
          const uint8_t* blk = row + (int64_t)(g * 32 + l) * Q3O_QBYTES;
          sc[l] = q3o_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
          for (int j = 0; j < 32; ++j) qT[j * 32 + l] = (float)(int8_t)blk[2 + j];
        } else {
          sc[l] = 0.0f;
          for (int j = 0; j < 32; ++j) qT[j * 32 + l] = 0.0f;
        }
        inner[l] = 0.0f;
      }
      const float* xg = c->xT + (size_t)g * 1024;
      for (int j = 0; j < 32; ++j)
        for (int l = 0; l < 32; ++l) inner[l] = fmaf(qT[j * 32 + l], xg[j * 32 + l], inner[l]);
      for (int l = 0; l < lanes; ++l) acc[l] = fmaf(sc[l], inner[l], acc[l]);
    }
    c->y[n] = q3o_f2h(butterfly_sum(acc));
  }
}

void q3o_gemv_q8_mlir(const uint8_t* w, const uint16_t* x, uint16_t* y, int N, int K) {
  const int nb = K / Q3O_QBLK;
  const int ngroups = (nb + 31) / 32;
  float* xf = (float*)malloc(sizeof(float) * (size_t)K);
  x_to_f32(x, xf, K);
  /* xT[g][j][l] = x[32*(32g+l) + j] so the inner loop runs over lanes */
  float* xT = (float*)calloc((size_t)ngroups * 32 * 32, sizeof(float));
  for (int b = 0; b < nb; ++b)
    for (int j = 0; j < 32; ++j) xT[((b / 32) * 32 + j) * 32 + (b % 32)] = xf[b * 32 + j];
  gemv_ctx c = {w, xf, xT, y, nb, ngroups};
  pool_for(N, gemv_q8_mlir_task, &c);
  free(xT);
  free(xf);
}

/* Q8_0 GEMV in the order of the reference's CUDA kernels
 * (kernels/cuda/dispatch_3.cu:33-47): lane l walks blocks b = l, l+32, ...;
 * per element acc = fma(scale*q, x, acc) (nvcc contracts
 * acc += scale*(float)q*x into one FFMA; scale*q is exact), then the butterfly. */
static void gemv_q8_cuda_task(void* vctx, int64_t n0, int64_t n1) {
  const gemv_ctx* c = (const gemv_ctx*)vctx;
  const int nb = c->nb;
  const int64_t rowbytes = (int64_t)nb * Q3O_QBYTES;
  for (int64_t n = n0; n < n1; ++n) {
    const uint8_t* row = c->w + n * rowbytes;
    float acc[32] = {0};
    for (int l = 0; l < 32; ++l) {
      float a = 0.0f;
      for (int b = l; b < nb; b += 32) {
        const uint8_t* blk = row + (int64_t)b * Q3O_QBYTES;
        const float s = q3o_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < 32; ++j) a = fmaf(s * (float)(int8_t)blk[2 + j], c->xf[b * 32 + j], a);
      }
      acc[l] = a;
    }
    c->y[n] = q3o_f2h(butterfly_sum(acc));
  }
}

void q3o_gemv_q8_cuda(const uint8_t* w, const uint16_t* x, uint16_t* y, int N, int K) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)K);
  x_to_f32(x, xf, K);
  gemv_ctx c = {w, xf, NULL, y, K / Q3O_QBLK, 0};
  pool_for(N, gemv_q8_cuda_task, &c);
  free(xf);
}

/* f16 GEMV of the vocab projection (kernels/cuda/dispatch_24.cu:32-45 and
 * kernels/mlir/dispatch_24_gpu.mlir:60-84): lane l accumulates
 * k = l, l+32, ... as an f32 fma chain, then the butterfly, f16 out. */
typedef struct {
  const uint16_t* w;
  const float* xf;
  uint16_t* y;
  int K;
} gemv16_ctx;

static void gemv_f16_task(void* vctx, int64_t n0, int64_t n1) {
  const gemv16_ctx* c = (const gemv16_ctx*)vctx;
  const int K = c->K;
  for (int64_t n = n0; n < n1; ++n) {
    const _Float16* row = (const _Float16*)(c->w + n * K);
    float acc[32] = {0};
    for (int i = 0; i < K; i += 32) {
      const int lanes = (K - i) < 32 ? (K - i) : 32;
      for (int l = 0; l < lanes; ++l) acc[l] = fmaf((float)row[i + l], c->xf[i + l], acc[l]);
    }
    c->y[n] = q3o_f2h(butterfly_sum(acc));
  }
}

void q3o_gemv_f16(const uint16_t* w, const uint16_t* x, uint16_t* y, int N, int K) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)K);
  x_to_f32(x, xf, K);
  gemv16_ctx c = {w, xf, y, K};
  pool_for(N, gemv_f16_task, &c);
  free(xf);
}

/* Tiled argmax of model/qwen3_full.mlir:1469-1509: strict ordered ">"
 * (arith.cmpf ogt) starting from -inf with index -1, so the lowest index of
 * the largest value wins, NaN and -inf are never chosen, and an input with no
 * value above -inf yields -1.  The two-phase tiling gives the same answer as
 * this single scan. */
int64_t q3o_argmax_f16(const uint16_t* v, int64_t n) {
  float best = -INFINITY;
  int64_t idx = -1;
  for (int64_t i = 0; i < n; ++i) {
    const float f = q3o_h2f(v[i]);
    if (f > best) {
      best = f;
      idx = i;
    }
  }
  return idx;
}

/* ---------------------------------------------------------------------- */
/* Small ops                                                              */
/* ---------------------------------------------------------------------- */

/* Sum of squares in lane order: lane l accumulates x[l+32i]^2 as an fma chain
 * over i, then the butterfly.  (The linalg reduction of
 * model/qwen3_full.mlir:135-143 fixes no order; this is the order the CUDA
 * kernels use.) */
static float sumsq_lanes(const float* xf, int n) {
  float acc[32] = {0};
  for (int i = 0; i < n; i += 32)
    for (int l = 0; l < 32 && i + l < n; ++l) acc[l] = fmaf(xf[i + l], xf[i + l], acc[l]);
  return butterfly_sum(acc);
}

/* rms_norm_1x1024 (model/qwen3_full.mlir:134-165):
 * r = sqrt(ss/n + eps); y = f16((x / r) * g) -- a divide by the root. */
void q3o_rmsnorm(const uint16_t* x, const uint16_t* g, uint16_t* y, int n) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)n);
  x_to_f32(x, xf, n);
  const float ss = sumsq_lanes(xf, n);
  const float r = sqrtf(ss / (float)n + kEps);
  for (int k = 0; k < n; ++k) y[k] = q3o_f2h((xf[k] / r) * q3o_h2f(g[k]));
  free(xf);
}

/* RoPE angles of rope_decode_q/k (model/qwen3_full.mlir:324-454):
 * theta_i = powf(1e6, -((2*i)/128)) * 1.0, a = f32(i32(pos)) * theta_i. */
void q3o_rope_table(int64_t n_pos, float* cos_t, float* sin_t) {
  for (int64_t p = 0; p < n_pos; ++p) {
    const float pf = (float)(int32_t)p;
    for (int i = 0; i < 64; ++i) {
      const float e = -((2.0f * (float)i) / 128.0f);
      const float th = powf(1.0e6f, e) * 1.0f;
      const float a = pf * th;
      cos_t[p * 64 + i] = cosf(a);
      sin_t[p * 64 + i] = sinf(a);
    }
  }
}

/* Per-head QK-RMSNorm (model/qwen3_full.mlir:646-702, f16 out) followed by
 * NeoX RoPE (model/qwen3_full.mlir:324-454, f16 out):
 *   y_i     = f16(x_i*c - x_{i+64}*s)
 *   y_{i+64} = f16(x_i*s + x_{i+64}*c)        (two products, one add; no fma) */
void q3o_qk_norm_rope(const uint16_t* x, const uint16_t* g, int n_heads, int64_t pos,
                      uint16_t* y) {
  float ct[64], st[64];
  {
    const float pf = (float)(int32_t)pos;
    for (int i = 0; i < 64; ++i) {
      const float e = -((2.0f * (float)i) / 128.0f);
      const float th = powf(1.0e6f, e) * 1.0f;
      const float a = pf * th;
      ct[i] = cosf(a);
      st[i] = sinf(a);
    }
  }
  for (int h = 0; h < n_heads; ++h) {
    float xf[Q3O_HD], nf[Q3O_HD];
    x_to_f32(x + h * Q3O_HD, xf, Q3O_HD);
    const float ss = sumsq_lanes(xf, Q3O_HD);
    const float r = sqrtf(ss / 128.0f + kEps);
    for (int k = 0; k < Q3O_HD; ++k)
      nf[k] = q3o_h2f(q3o_f2h((xf[k] / r) * q3o_h2f(g[k])));
    for (int i = 0; i < 64; ++i) {
      const float a = nf[i], b = nf[i + 64];
      y[h * Q3O_HD + i] = q3o_f2h(a * ct[i] - b * st[i]);
      y[h * Q3O_HD + i + 64] = q3o_f2h(a * st[i] + b * ct[i]);
    }
  }
}

/* SwiGLU in f16 arithmetic (model/qwen3_full.mlir:824-839): every op rounds
 * to f16; math.exp on f16 is evaluated in f32 and rounded. */
void q3o_swiglu(const uint16_t* gate_up, uint16_t* out, int n) {
  for (int i = 0; i < n; ++i) {
    const float g = q3o_h2f(gate_up[i]);
    const float u = q3o_h2f(gate_up[n + i]);
    const float e = q3o_h2f(q3o_f2h(q3o_expf(-g)));
    const float den = q3o_h2f(q3o_f2h(1.0f + e));
    const float sig = q3o_h2f(q3o_f2h(1.0f / den));
    const float silu = q3o_h2f(q3o_f2h(g * sig));
    out[i] = q3o_f2h(silu * u);
  }
}

/* Residual add in f16 (model/qwen3_full.mlir:801-805, :858-862). */
void q3o_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* y, int n) {
  for (int i = 0; i < n; ++i) y[i] = q3o_f2h(q3o_h2f(a[i]) + q3o_h2f(b[i]));
}

/* GQA decode attention (model/qwen3_full.mlir:456-530): q head h reads kv
 * head h/2; out = softmax(scale * q.k_t) . v over keys t = 0..T-1, all keys
 * visible (decode mask is all-true), f32 inside, f16 out.  The softmax is
 * evaluated in the chunked order of the CUDA kernel (IREE's own order is not
 * pinned): keys fall into chunks of 32; a chunk yields (m, l, o[128]) with
 *   s_t = (fma chain of q_d*k_td over d) * scale,  m = max s_t,
 *   p_t = exp(s_t - m),  l = butterfly sum of p_t,
 *   o_d = fma chain of p_t*v_td over t in key order;
 * chunks are folded in two levels -- left to right within each group of
 * Q3O_ATT_GROUP consecutive chunks (one CTA of the kernel), then the group
 * results left to right -- each fold step being
 *   m = max(ma, mb), a = exp(ma - m), b = exp(mb - m),
 *   l = fma(lb, b, la*a),  o_d = fma(ob_d, b, oa_d*a);
 * finally out_d = f16(o_d / l).  With T <= 256 there is one group and the
 * fold is a plain left-to-right fold of the chunks. */
typedef struct {
  float m, l;
  float o[Q3O_HD];
} att_part;

static void att_merge(att_part* a, const att_part* b) {
  const float m = fmaxf(a->m, b->m);
  const float ea = q3o_expf(a->m - m);
  const float eb = q3o_expf(b->m - m);
  a->l = fmaf(b->l, eb, a->l * ea);
  for (int d = 0; d < Q3O_HD; ++d) a->o[d] = fmaf(b->o[d], eb, a->o[d] * ea);
  a->m = m;
}

/* One chunk of 32 keys (c*32 .. c*32+31, those < T) of kv head kvh: the
 * partial (m, l, o) of the q head held in qf (f32 of the f16 values). */
static void att_chunk(const float* qf, const uint16_t* kc, const uint16_t* vc, int64_t slot0,
                      int kvh, int64_t c, int64_t T, att_part* out) {
  const int64_t row = (int64_t)Q3O_NKV * Q3O_HD;
  float s[32], p[32];
  int valid = 0;
  for (int l = 0; l < 32; ++l) {
    const int64_t t = c * 32 + l;
    if (t < T) {
      const uint16_t* k = kc + (slot0 + t) * row + kvh * Q3O_HD;
      float a = 0.0f;
      for (int d = 0; d < Q3O_HD; ++d) a = fmaf(qf[d], q3o_h2f(k[d]), a);
      s[l] = a * kAttnScale;
      ++valid;
    } else {
      s[l] = -INFINITY;
    }
  }
  float m = -INFINITY;
  for (int l = 0; l < 32; ++l) m = fmaxf(m, s[l]);
  for (int l = 0; l < 32; ++l) p[l] = (l < valid) ? q3o_expf(s[l] - m) : 0.0f;
  out->m = m;
  out->l = butterfly_sum(p);
  for (int d = 0; d < Q3O_HD; ++d) out->o[d] = 0.0f;
  for (int l = 0; l < valid; ++l) {
    const uint16_t* v = vc + (slot0 + c * 32 + l) * row + kvh * Q3O_HD;
    for (int d = 0; d < Q3O_HD; ++d) out->o[d] = fmaf(p[l], q3o_h2f(v[d]), out->o[d]);
  }
}

void q3o_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int64_t slot0,
                   int64_t T, uint16_t* out) {
  const int64_t nchunks = (T + Q3O_ATT_CHUNK - 1) / Q3O_ATT_CHUNK;
  for (int h = 0; h < Q3O_NQ; ++h) {
    const int kvh = h / 2;
    float qf[Q3O_HD];
    x_to_f32(q + h * Q3O_HD, qf, Q3O_HD);
    att_part total, group, chunk;
    for (int64_t c = 0; c < nchunks; ++c) {
      att_chunk(qf, kc, vc, slot0, kvh, c, T, &chunk);
      if (c % Q3O_ATT_GROUP == 0)
        group = chunk;
      else
        att_merge(&group, &chunk);
      if (c % Q3O_ATT_GROUP == Q3O_ATT_GROUP - 1 || c == nchunks - 1) {
        if (c < Q3O_ATT_GROUP)
          total = group;
        else
          att_merge(&total, &group);
      }
    }
    for (int d = 0; d < Q3O_HD; ++d) out[h * Q3O_HD + d] = q3o_f2h(total.o[d] / total.l);
  }
}

/* The fused engine's attention (k_fused_attn).  Chunks of 8 keys; key t's
 * dot is split in four quarters of 32 dims (fma chains), combined as
 * (a0 + a1) + (a2 + a3), times rsqrt(128); per chunk m = max s_t,
 * p_t = exp(s_t - m) (0 past the end), l = ((p0 + p1) + (p2 + p3)) +
 * ((p4 + p5) + (p6 + p7)), o_d = fma chain of p_t * v_td over t.  Chunk c
 * belongs to cluster rank c % 16 as local chunk j = c / 16, handled by warp
 * j % 8 in pass j / 8; a warp folds its chunks in pass order with the
 * pairwise merge of q3o_attention (att_merge); rank r folds its 8 warps
 * (M_r = max m_w, e_w = exp(m_w - M_r), fma chains of l_w * e_w and
 * o_w * e_w over w, warps without chunks skipped), the cluster folds the
 * ranks the same way (ranks without chunks skipped) and out = f16(O / L). */
static void att_chunk8(const float* qf, const uint16_t* kc, const uint16_t* vc, int64_t slot0,
                       int kvh, int64_t c, int64_t T, att_part* out) {
  const int64_t row = (int64_t)Q3O_NKV * Q3O_HD;
  float s[8], p[8];
  for (int l = 0; l < 8; ++l) {
    const int64_t t = c * 8 + l;
    if (t < T) {
      const uint16_t* k = kc + (slot0 + t) * row + kvh * Q3O_HD;
      float a[4];
      for (int q = 0; q < 4; ++q) {
        float acc = 0.0f;
        for (int d = 32 * q; d < 32 * q + 32; ++d) acc = fmaf(qf[d], q3o_h2f(k[d]), acc);
        a[q] = acc;
      }
      s[l] = ((a[0] + a[1]) + (a[2] + a[3])) * kAttnScale;
    } else {
      s[l] = -INFINITY;
    }
  }
  float m = -INFINITY;
  for (int l = 0; l < 8; ++l) m = fmaxf(m, s[l]);
  for (int l = 0; l < 8; ++l) p[l] = (c * 8 + l < T) ? q3o_expf(s[l] - m) : 0.0f;
  out->m = m;
  out->l = ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
  for (int d = 0; d < Q3O_HD; ++d) out->o[d] = 0.0f;
  for (int l = 0; l < 8 && c * 8 + l < T; ++l) {
    const uint16_t* v = vc + (slot0 + c * 8 + l) * row + kvh * Q3O_HD;
    for (int d = 0; d < Q3O_HD; ++d) out->o[d] = fmaf(p[l], q3o_h2f(v[d]), out->o[d]);
  }
}

/* max-first fold of n partials (those with have[i]) into *out */
static void att_fold_maxfirst(const att_part* p, const int* have, int n, att_part* out) {
  out->m = -INFINITY;
  out->l = 0.0f;
  for (int d = 0; d < Q3O_HD; ++d) out->o[d] = 0.0f;
  for (int i = 0; i < n; ++i)
    if (have[i]) out->m = fmaxf(out->m, p[i].m);
  for (int i = 0; i < n; ++i) {
    if (!have[i]) continue;
    const float e = q3o_expf(p[i].m - out->m);
    out->l = fmaf(p[i].l, e, out->l);
    for (int d = 0; d < Q3O_HD; ++d) out->o[d] = fmaf(p[i].o[d], e, out->o[d]);
  }
}

void q3o_attention_fused(const uint16_t* q, const uint16_t* kc, const uint16_t* vc,
                         int64_t slot0, int64_t T, uint16_t* out) {
  enum { R = Q3O_FUSED_CLUSTER, W = 8 };
  const int64_t nchunks = (T + 7) / 8;
  for (int h = 0; h < Q3O_NQ; ++h) {
    const int kvh = h / 2;
    float qf[Q3O_HD];
    x_to_f32(q + h * Q3O_HD, qf, Q3O_HD);
    att_part rk[R];
    int rk_have[R];
    for (int r = 0; r < R; ++r) {
      att_part wp[W];
      int w_have[W];
      for (int w = 0; w < W; ++w) {
        w_have[w] = 0;
        for (int64_t j = w; r + (int64_t)R * j < nchunks; j += W) {
          att_part ch;
          att_chunk8(qf, kc, vc, slot0, kvh, r + (int64_t)R * j, T, &ch);
          if (!w_have[w])
            wp[w] = ch;
          else
            att_merge(&wp[w], &ch);
          w_have[w] = 1;
        }
      }
      att_fold_maxfirst(wp, w_have, W, &rk[r]);
      rk_have[r] = r < nchunks;
    }
    att_part tot;
    att_fold_maxfirst(rk, rk_have, R, &tot);
    for (int d = 0; d < Q3O_HD; ++d) out[h * Q3O_HD + d] = q3o_f2h(tot.o[d] / tot.l);
  }
}

/* The fused engine's RMSNorm of the residual stream: the 16 ranks of a
 * cluster each rebuild 64 elements (rank r: 64r .. 64r+63, lane t of 16:
 * 4t .. 4t+3); a lane's sum of squares is an fma chain over its 4 elements,
 * the rank's is the butterfly over its 16 lanes (offsets 8, 4, 2, 1), and
 * ss = ((ss_0 + ss_1) + ...) + ss_15.  Then r = sqrt(ss/1024 + eps) and
 * y = f16((x / r) * g) as in q3o_rmsnorm. */
static void rmsnorm_fused(const uint16_t* x, const uint16_t* g, uint16_t* y) {
  float xf[Q3O_DIM];
  x_to_f32(x, xf, Q3O_DIM);
  float ss = 0.0f;
  for (int r = 0; r < 16; ++r) {
    float a[16];
    for (int t = 0; t < 16; ++t) {
      float acc = 0.0f;
      for (int i = 0; i < 4; ++i) {
        const float v = xf[64 * r + 4 * t + i];
        acc = fmaf(v, v, acc);
      }
      a[t] = acc;
    }
    for (int off = 8; off > 0; off >>= 1) {
      float b[16];
      for (int t = 0; t < 16; ++t) b[t] = a[t] + a[t ^ off];
      for (int t = 0; t < 16; ++t) a[t] = b[t];
    }
    ss = r == 0 ? a[0] : ss + a[0];
  }
  const float rn = sqrtf(ss / (float)Q3O_DIM + kEps);
  for (int k = 0; k < Q3O_DIM; ++k) y[k] = q3o_f2h((xf[k] / rn) * q3o_h2f(g[k]));
}

/* The fused engine's split GEMV (k_fused_attn's W_o slice, k_fused_ffn's
 * W_down slice): K is cut into nparts slices of bpp = K/32/nparts blocks;
 * in slice p, lane sub (0..3) accumulates blocks p*bpp + sub*bpp/4 + i
 * (i < bpp/4) as acc = fma(scale, inner, acc) with inner the fma chain of
 * q_j * x_j over j; the slice partial is (a0 + a1) + (a2 + a3); the row is
 * f16 of the partials summed in slice order. */
typedef struct {
  const uint8_t* w;
  const float* xf;
  uint16_t* y;
  int nb, nparts;
} split_ctx;

static void gemv_q8_split_task(void* vctx, int64_t n0, int64_t n1) {
  const split_ctx* c = (const split_ctx*)vctx;
  const int bpp = c->nb / c->nparts, bps = bpp / 4;
  for (int64_t n = n0; n < n1; ++n) {
    const uint8_t* row = c->w + n * (int64_t)c->nb * Q3O_QBYTES;
    float total = 0.0f;
    for (int p = 0; p < c->nparts; ++p) {
      float a[4];
      for (int sub = 0; sub < 4; ++sub) {
        float acc = 0.0f;
        for (int i = 0; i < bps; ++i) {
          const int b = p * bpp + sub * bps + i;
          const uint8_t* blk = row + (int64_t)b * Q3O_QBYTES;
          const float sc = q3o_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
          float inner = 0.0f;
          for (int j = 0; j < 32; ++j) inner = fmaf((float)(int8_t)blk[2 + j], c->xf[b * 32 + j], inner);
          acc = fmaf(sc, inner, acc);
        }
        a[sub] = acc;
      }
      const float part = (a[0] + a[1]) + (a[2] + a[3]);
      total = p == 0 ? part : total + part;
    }
    c->y[n] = q3o_f2h(total);
  }
}

void q3o_gemv_q8_split(const uint8_t* w, const uint16_t* x, uint16_t* y, int N, int K,
                       int nparts) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)K);
  x_to_f32(x, xf, K);
  split_ctx c = {w, xf, y, K / Q3O_QBLK, nparts};
  pool_for(N, gemv_q8_split_task, &c);
  free(xf);
}

/* ---------------------------------------------------------------------- */
/* Layer, step, generate                                                  */
/* ---------------------------------------------------------------------- */

static const int64_t kBplQ = 2228224, kBplKV = 1114112, kBplO = 2228224, kBplGU = 6684672,
                     kBplD = 3342336;

/* transformer_layer_decode_static (model/qwen3_full.mlir:751-864) with the
 * attention block of :591-748.  The new K (normed, roped) and V are written
 * at slot layer*S + pos first; attending over slots layer*S + 0..pos is the
 * same as the reference's concat of the cached ctx slice with the new row
 * (:715-720) because ctx == pos on every call path (:1431-1523, :1555-1566). */
void q3o_layer(const q3o_weights* w, int layer, uint16_t* x, int64_t pos, uint16_t* kc,
               uint16_t* vc, int64_t S) {
  uint16_t xn[Q3O_DIM], q[2048], k[1024], v[1024], qn[2048], kn[1024], att[2048], o[1024],
      h1[1024], hn[1024], gu[6144], act[3072], d[1024];
  const int fused = w->order == Q3O_ORDER_FUSED;
  if (fused)
    rmsnorm_fused(x, w->attn_norm + layer * Q3O_DIM, xn);
  else
    q3o_rmsnorm(x, w->attn_norm + layer * Q3O_DIM, xn, Q3O_DIM);
  q3o_gemv_q8_mlir(w->q8_q + layer * kBplQ, xn, q, 2048, 1024);
  q3o_gemv_q8_mlir(w->q8_k + layer * kBplKV, xn, k, 1024, 1024);
  q3o_gemv_q8_mlir(w->q8_v + layer * kBplKV, xn, v, 1024, 1024);
  q3o_qk_norm_rope(q, w->q_norm + layer * Q3O_HD, Q3O_NQ, pos, qn);
  q3o_qk_norm_rope(k, w->k_norm + layer * Q3O_HD, Q3O_NKV, pos, kn);
  const int64_t slot = (int64_t)layer * S + pos;
  memcpy(kc + slot * 1024, kn, sizeof(kn));
  memcpy(vc + slot * 1024, v, sizeof(v));
  if (fused)
    q3o_attention_fused(qn, kc, vc, (int64_t)layer * S, pos + 1, att);
  else
    q3o_attention(qn, kc, vc, (int64_t)layer * S, pos + 1, att);
  if (fused)
    q3o_gemv_q8_split(w->q8_o + layer * kBplO, att, o, 1024, 2048, 8);
  else
    q3o_gemv_q8_mlir(w->q8_o + layer * kBplO, att, o, 1024, 2048);
  q3o_add_f16(x, o, h1, Q3O_DIM);
  if (fused)
    rmsnorm_fused(h1, w->ffn_norm + layer * Q3O_DIM, hn);
  else
    q3o_rmsnorm(h1, w->ffn_norm + layer * Q3O_DIM, hn, Q3O_DIM);
  q3o_gemv_q8_mlir(w->q8_gate_up + layer * kBplGU, hn, gu, 6144, 1024);
  q3o_swiglu(gu, act, Q3O_FFN);
  if (fused)
    q3o_gemv_q8_split(w->q8_down + layer * kBplD, act, d, 1024, 3072, 8);
  else
    q3o_gemv_q8_mlir(w->q8_down + layer * kBplD, act, d, 1024, 3072);
  q3o_add_f16(h1, d, x, Q3O_DIM);
}

/* One decode step = the body of @generate's inner loop
 * (model/qwen3_full.mlir:1431-1509): embedding gather, the layers, final
 * RMSNorm with output_norm, f16 vocab GEMV and the tiled argmax. */
int64_t q3o_decode_step(const q3o_weights* w, int64_t token, int64_t pos, uint16_t* kc,
                        uint16_t* vc, int64_t S, uint16_t* logits, int want_logits) {
  uint16_t x[Q3O_DIM], xn[Q3O_DIM];
  memcpy(x, w->token_embd + token * Q3O_DIM, sizeof(x));
  for (int l = 0; l < w->n_layers; ++l) q3o_layer(w, l, x, pos, kc, vc, S);
  if (!want_logits) return -1;
  q3o_rmsnorm(x, w->output_norm, xn, Q3O_DIM);
  q3o_gemv_f16(w->output_T, xn, logits, Q3O_VOCAB, Q3O_DIM);
  return q3o_argmax_f16(logits, Q3O_VOCAB);
}

/* @run (model/qwen3_full.mlir:2113-2167) with the prompt ingested through the
 * decode path as @prefill_all does (:1541-1570), then @generate (:1396-1534):
 * groups of 4 tokens, and the loop stops when the LAST token of a group is
 * eos (a mid-group eos does not stop it).  The first token (argmax of the last
 * prompt step) is fed at position n_prompt and is not itself returned, as in
 * the reference.  Returns the number of generated tokens.
 * force_tokens (optional): teacher forcing -- step i feeds force_tokens[i]
 * instead of its own argmax (the argmax is still reported).  n_prompt >= 1. */
int64_t q3o_generate(const q3o_weights* w, const int64_t* prompt, int64_t n_prompt,
                     int64_t max_gen, int64_t eos, uint16_t* kc, uint16_t* vc, int64_t S,
                     int64_t* out_tokens, const int64_t* force_tokens) {
  if (n_prompt < 1) return -1;
  uint16_t* logits = (uint16_t*)malloc(sizeof(uint16_t) * Q3O_VOCAB);
  int64_t tok = -1;
  for (int64_t i = 0; i < n_prompt; ++i)
    tok = q3o_decode_step(w, prompt[i], i, kc, vc, S, logits, i + 1 == n_prompt);
  int64_t pos = n_prompt, count = 0;
  int not_eos = 1;
  while (count < max_gen && not_eos) {
    const int64_t rem = max_gen - count;
    const int64_t batch = rem < 4 ? rem : 4;
    for (int64_t b = 0; b < batch; ++b) {
      const int64_t next = q3o_decode_step(w, tok, pos, kc, vc, S, logits, 1);
      out_tokens[count] = next;
      tok = force_tokens ? force_tokens[count] : next;
      ++count;
      ++pos;
    }
    not_eos = (tok != eos);
  }
  free(logits);
  return count;
}

int q3o_num_threads(void) {
  pool_start();
  return g_pool.nthreads;
}

/* Takes effect only before the pool's first use (the pool is persistent). */
void q3o_set_num_threads(int n) {
  if (!g_pool.started) g_want_threads = n;
}
