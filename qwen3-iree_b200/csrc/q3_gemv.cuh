// q3_gemv.cuh -- batch-1 GEMV kernels for sm_100a.
//
//   * Q8_0 fused dequant + GEMV (replaces kernels/cuda/dispatch_{3,4,12,18,20}.cu
//     and their GPU-dialect twins), with optional fused RMSNorm prologue,
//     residual-add epilogue, or SwiGLU epilogue over gate/up row pairs;
//   * f16 vocab GEMV (replaces kernels/cuda/dispatch_24.cu) fused with the
//     tiled argmax of model/qwen3_full.mlir:1469-1509.
//
// Data path: a producer warp streams tiles of 8 weight rows from HBM into a
// ring of shared-memory stages with 1-D bulk copies (cp.async.bulk, TMA
// engine, completion on mbarriers); eight consumer warps compute from shared
// memory.  Weight rows are used in the reference's native layout (Q8_0 rows
// of K/32 34-byte blocks, f16 rows), 16-byte aligned row starts.
//
// Lane mapping = the reference's: warp per row; for Q8_0 lane l owns blocks
// l, l+32, ... (the input slice for those blocks lives in registers); for f16
// lane l owns k = l, l+32, ....  Summation orders therefore match the
// reference kernels exactly (see q3_common.cuh).
#pragma once

#include "q3_common.cuh"

namespace q3 {

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kTileRows = 8;
constexpr int kMaxSeg = 32;

enum GemvOrder : int { kOrderMlir = 0, kOrderCuda = 1 };
enum GemvMode : int { kModePlain = 0, kModeNormIn = 1, kModeResid = 2, kModeSwiglu = 3 };

// Device-resident decode state of one sequence (read by the step kernels).
struct SeqState {
  int64_t pos;       // position of the token fed in the current step
  int64_t n_prompt;  // prompt length; steps at pos >= n_prompt produce output
  int64_t n_gen;     // generated tokens so far
  int64_t max_gen;
  int64_t eos;
  int32_t stop;      // set once the reference's end rule fired
  int32_t pad;
};

struct Q8Seg {
  const uint8_t* w;   // first row of this segment
  const uint16_t* x;  // input (f16 bits); with kModeNormIn, the un-normalised input
  uint16_t* y;        // output rows of this segment
  const uint16_t* r;  // residual rows (kModeResid) aligned with y
};

struct Q8GemvArgs {
  Q8Seg seg[kMaxSeg];
  int nseg;
  int seg_rows;          // rows per segment (multiple of 8)
  int K;                 // multiple of 256, <= 3072
  int64_t up_off_bytes;  // kModeSwiglu: byte offset from a gate row to its up row
  const uint16_t* norm_g;  // kModeNormIn: RMSNorm gamma [K]
  // Layer-0 embedding gather (kModeNormIn only): when tokens != nullptr the
  // input is row tokens[seq->pos] of embd, and CTA 0 also stores it to embed_out.
  const int64_t* tokens;
  const SeqState* seq;
  int64_t S;             // positions the token table covers (tokens has S + 1 entries)
  const uint16_t* embd;
  uint16_t* embed_out;
  SeqState* advance;     // if set, pos += 1 (the step's last kernel, prompt ingestion)
  int* err;
  int nstages;
  unsigned long long* trace;  // optional launch timing record (4 values)
  // Optional L2 prefetch of the next launch's weights (up to 3 ranges, 16-byte
  // aligned, sizes multiples of 16), split across this launch's CTAs and issued
  // before the dependency wait, so that next launch's late-starting CTAs find
  // their tiles in L2.
  const uint8_t* pf_ptr[3];
  uint32_t pf_bytes[3];
};

// This CTA's share of the L2 prefetch ranges.
__device__ __forceinline__ void q8_prefetch_next(const Q8GemvArgs& a) {
#pragma unroll
  for (int r = 0; r < 3; ++r) {
    const uint32_t n = a.pf_bytes[r];
    if (n == 0) continue;
    const uint32_t share = ((n + gridDim.x - 1) / gridDim.x + 15u) & ~15u;
    const uint32_t off = blockIdx.x * share;
    if (off < n) bulk_prefetch_l2(a.pf_ptr[r] + off, n - off < share ? n - off : share);
  }
}

// --------------------------------------------------------------------------
// Input slices in registers
// --------------------------------------------------------------------------
template <int G>
__device__ __forceinline__ void load_x_blocks(const uint16_t* x, int nb, int lane,
                                              uint32_t (&xr)[G][16]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int b = lane + 32 * g;
    if (b < nb) {
      const uint4* p = reinterpret_cast<const uint4*>(x + 32 * b);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const uint4 t = p[v];
        xr[g][4 * v + 0] = t.x;
        xr[g][4 * v + 1] = t.y;
        xr[g][4 * v + 2] = t.z;
        xr[g][4 * v + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) xr[g][i] = 0u;
    }
  }
}

// RMSNorm of model/qwen3_full.mlir:134-165 evaluated per warp:
// ss in lane-strided fma order + butterfly; r = sqrt(ss/K + eps).
__device__ __forceinline__ float rms_denominator(const uint16_t* x, int K, int lane) {
  float ss = 0.0f;
  for (int k = lane; k < K; k += 32) {
    const float v = h2f(x[k]);
    ss = __fmaf_rn(v, v, ss);
  }
  ss = warp_sum(ss);
  return __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), kEps));
}

__device__ __forceinline__ uint16_t rms_apply(uint16_t x, uint16_t g, float r) {
  return f2h(__fmul_rn(__fdiv_rn(h2f(x), r), h2f(g)));
}

template <int G>
__device__ __forceinline__ void load_x_blocks_norm(const uint16_t* x, const uint16_t* gamma,
                                                   int K, int lane, uint32_t (&xr)[G][16]) {
  const float r = rms_denominator(x, K, lane);
  const int nb = K / kQBlk;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int b = lane + 32 * g;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      uint32_t v = 0u;
      if (b < nb) {
        const int k = 32 * b + 2 * i;
        v = (uint32_t)rms_apply(x[k], gamma[k], r) |
            ((uint32_t)rms_apply(x[k + 1], gamma[k + 1], r) << 16);
      }
      xr[g][i] = v;
    }
  }
}

// Barrier over the 256 consumer threads (warps 0-7) only: the producer warp
// never joins it.
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// The same RMSNorm computed once per CTA by the 256 consumer threads into
// shared memory: x staged in xs, ss in warp 0's lane-strided order, then
// xs[k] = f16((x_k / r) * g_k).  x 16-byte aligned, K a multiple of 8.
__device__ __forceinline__ void cta_rmsnorm_to_smem(const uint16_t* x, const uint16_t* g, int K,
                                                    uint16_t* xs, float* rs) {
  const int tid = threadIdx.x;
  for (int i = tid; i < K / 8; i += 256)
    reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(x)[i];
  consumer_sync();
  if (tid < 32) {
    float ss = 0.0f;
    for (int k = tid; k < K; k += 32) {
      const float v = h2f(xs[k]);
      ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if (tid == 0) *rs = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), kEps));
  }
  consumer_sync();
  const float r = *rs;
  for (int k = tid; k < K; k += 256) xs[k] = rms_apply(xs[k], g[k], r);
  consumer_sync();
}

// The same RMSNorm with this thread's gamma values already in registers
// (gr[i] = g[threadIdx.x + 256 i], loaded before the wait on the previous
// kernel: gamma is a constant).  KMAX bounds K (a multiple of 256).
template <int KMAX>
__device__ __forceinline__ void load_gamma_regs(const uint16_t* g, int K,
                                                uint16_t (&gr)[KMAX / 256]) {
#pragma unroll
  for (int i = 0; i < KMAX / 256; ++i) {
    const int k = threadIdx.x + 256 * i;
    gr[i] = k < K ? g[k] : (uint16_t)0;
  }
}
// x == nullptr: xs already holds the input (staged by the caller).
template <int KMAX>
__device__ __forceinline__ void cta_rmsnorm_to_smem_g(const uint16_t* x,
                                                      const uint16_t (&gr)[KMAX / 256], int K,
                                                      uint16_t* xs, float* rs) {
  const int tid = threadIdx.x;
  if (x != nullptr)
    for (int i = tid; i < K / 8; i += 256)
      reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(x)[i];
  consumer_sync();
  if (tid < 32) {
    float ss = 0.0f;
    for (int k = tid; k < K; k += 32) {
      const float v = h2f(xs[k]);
      ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if (tid == 0) *rs = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), kEps));
  }
  consumer_sync();
  const float r = *rs;
#pragma unroll
  for (int i = 0; i < KMAX / 256; ++i) {
    const int k = tid + 256 * i;
    if (k < K) xs[k] = rms_apply(xs[k], gr[i], r);
  }
  consumer_sync();
}

template <int G>
__device__ __forceinline__ void h2_to_f32(const uint32_t (&xr)[G][16], float (&xf)[G][32]) {
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      xf[g][2 * i] = h2f((uint16_t)(xr[g][i] & 0xffffu));
      xf[g][2 * i + 1] = h2f((uint16_t)(xr[g][i] >> 16));
    }
}

// Dot of one Q8_0 row held in shared memory at byte address `row`.
template <int G, int ORDER>
__device__ __forceinline__ float q8_row_dot(uint32_t row, int nb, int lane,
                                            const uint32_t (&xr)[G][16]) {
  float acc = 0.0f;
  if constexpr (ORDER == kOrderMlir) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int b = lane + 32 * g;
      if (b < nb) {
        const Q8BlockWords bw = q8_load_block(row + (uint32_t)(kQBytes * b));
        acc = q8_block_dot_mlir(bw, xr[g], acc);
      }
    }
  } else {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int b = lane + 32 * g;
      if (b < nb) {
        float xf[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          xf[2 * i] = h2f((uint16_t)(xr[g][i] & 0xffffu));
          xf[2 * i + 1] = h2f((uint16_t)(xr[g][i] >> 16));
        }
        const Q8BlockWords bw = q8_load_block(row + (uint32_t)(kQBytes * b));
        acc = q8_block_dot_cuda(bw, xf, acc);
      }
    }
  }
  return warp_sum(acc);
}

// --------------------------------------------------------------------------
// x staged once per CTA as f32 in shared memory (k_gemv_q8)
// --------------------------------------------------------------------------
// Block b's 32 values sit at floats [36 b, 36 b + 32) (144 bytes a block).
// A lane reads its own block b = lane + 32 g as 8 float4; at float4 i that is
// 16-byte bank group (9 b + i) mod 8, distinct across the 8 lanes of a
// quarter warp, so the reads are conflict-free.  f16 -> f32 is exact, so the
// row dots see the same operand values as with f16 x.
constexpr int kXfStride = 36;

__device__ __forceinline__ int xf_index(int k) { return (k >> 5) * kXfStride + (k & 31); }

// The f16 copy for rows kept as half2: block b's 32 values at halves
// [40 b, 40 b + 32) (80 bytes a block), read as 4 uint4 per lane; at uint4 i
// that is bank group (5 b + i) mod 8, again distinct across a quarter warp.
constexpr int kXhStride = 40;

__device__ __forceinline__ int xh_index(int k) { return (k >> 5) * kXhStride + (k & 31); }

// x (f16, K a multiple of 8, 16-byte aligned) -> xf (F32) and/or xh (F16) by
// the 256 consumer threads; ends with a consumer barrier.
template <bool F32, bool F16>
__device__ __forceinline__ void stage_x(const uint16_t* x, int K, float* xf, uint16_t* xh) {
  for (int i = threadIdx.x; i < K / 8; i += 256) {
    const uint4 v = reinterpret_cast<const uint4*>(x)[i];
    if constexpr (F32) {
      float* d = xf + xf_index(8 * i);
      *reinterpret_cast<float4*>(d) =
          make_float4(h2f((uint16_t)(v.x & 0xffffu)), h2f((uint16_t)(v.x >> 16)),
                      h2f((uint16_t)(v.y & 0xffffu)), h2f((uint16_t)(v.y >> 16)));
      *reinterpret_cast<float4*>(d + 4) =
          make_float4(h2f((uint16_t)(v.z & 0xffffu)), h2f((uint16_t)(v.z >> 16)),
                      h2f((uint16_t)(v.w & 0xffffu)), h2f((uint16_t)(v.w >> 16)));
    }
    if constexpr (F16) *reinterpret_cast<uint4*>(xh + xh_index(8 * i)) = v;
  }
  consumer_sync();
}

__device__ __forceinline__ void stage_x_f32(const uint16_t* x, int K, float* xf) {
  stage_x<true, false>(x, K, xf, nullptr);
}

// RMSNorm into xf and/or xh: the same operations and order as
// cta_rmsnorm_to_smem_g (sum of squares in warp 0's lane-strided order,
// x_k / r * g_k rounded to f16), the normalised values stored as f32 / f16.
template <int KMAX, bool F32, bool F16>
__device__ __forceinline__ void cta_rmsnorm_to_x(const uint16_t* x,
                                                 const uint16_t (&gr)[KMAX / 256], int K,
                                                 float* xf, uint16_t* xh, float* rs) {
  const int tid = threadIdx.x;
  stage_x<F32, F16>(x, K, xf, xh);
  if (tid < 32) {
    float ss = 0.0f;
    for (int k = tid; k < K; k += 32) {
      const float v = F32 ? xf[xf_index(k)] : h2f(xh[xh_index(k)]);
      ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if (tid == 0) *rs = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), kEps));
  }
  consumer_sync();
  const float r = *rs;
#pragma unroll
  for (int i = 0; i < KMAX / 256; ++i) {
    const int k = tid + 256 * i;
    if (k < K) {
      const float v = F32 ? xf[xf_index(k)] : h2f(xh[xh_index(k)]);
      const uint16_t nh = f2h(__fmul_rn(__fdiv_rn(v, r), h2f(gr[i])));
      if constexpr (F32) xf[xf_index(k)] = h2f(nh);
      if constexpr (F16) xh[xh_index(k)] = nh;
    }
  }
  consumer_sync();
}

template <int KMAX>
__device__ __forceinline__ void cta_rmsnorm_to_xf(const uint16_t* x,
                                                  const uint16_t (&gr)[KMAX / 256], int K,
                                                  float* xf, float* rs) {
  cta_rmsnorm_to_x<KMAX, true, false>(x, gr, K, xf, nullptr, rs);
}

// Dot of one Q8_0 row (shared byte address `row`) with x staged in xf, in
// the same per-block orders as q8_row_dot: MLIR, inner = fma chain of
// q_j * x_j over j then acc = fma(scale, inner, acc); CUDA, acc = fma(scale *
// q_j, x_j, acc) per element.  int8 -> f32 by the exact byte-perm offset.
template <int G, int ORDER>
__device__ __forceinline__ float q8_row_dot_xf(uint32_t row, int nb, int lane, const float* xf) {
  float acc = 0.0f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int b = lane + 32 * g;
    if (b < nb) {
      const Q8BlockWords bw = q8_load_block(row + (uint32_t)(kQBytes * b));
      const float4* xb = reinterpret_cast<const float4*>(xf + b * kXfStride);
      if constexpr (ORDER == kOrderMlir) {
        float inner = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 xv = xb[i];
          float f[4];
          q8x4_to_f32(bw.q[i], f);
          inner = __fmaf_rn(f[0], xv.x, inner);
          inner = __fmaf_rn(f[1], xv.y, inner);
          inner = __fmaf_rn(f[2], xv.z, inner);
          inner = __fmaf_rn(f[3], xv.w, inner);
        }
        acc = __fmaf_rn(h2f((uint16_t)bw.scale16), inner, acc);
      } else {
        const float sc = h2f((uint16_t)bw.scale16);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 xv = xb[i];
          float f[4];
          q8x4_to_f32(bw.q[i], f);
          acc = __fmaf_rn(__fmul_rn(sc, f[0]), xv.x, acc);
          acc = __fmaf_rn(__fmul_rn(sc, f[1]), xv.y, acc);
          acc = __fmaf_rn(__fmul_rn(sc, f[2]), xv.z, acc);
          acc = __fmaf_rn(__fmul_rn(sc, f[3]), xv.w, acc);
        }
      }
    }
  }
  return warp_sum(acc);
}

// --------------------------------------------------------------------------
// Ring of shared-memory stages fed by the producer warp
// --------------------------------------------------------------------------
struct Ring {
  uint8_t* buf;
  uint64_t* full;
  uint64_t* empty;
  uint32_t stage_bytes;
  int ns;
};

__device__ __forceinline__ Ring ring_setup(uint8_t* smem, int ns, uint32_t stage_bytes,
                                           int consumers) {
  Ring r;
  r.full = reinterpret_cast<uint64_t*>(smem);
  r.empty = r.full + ns;
  r.buf = smem + 128 * ((16 * ns + 127) / 128);
  r.stage_bytes = stage_bytes;
  r.ns = ns;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&r.full[s], 1);
      mbar_init(&r.empty[s], consumers);
    }
    fence_mbar_init();
  }
  __syncthreads();
  return r;
}

__host__ __device__ inline size_t ring_smem_bytes(int ns, uint32_t stage_bytes) {
  return 128 * ((16 * (size_t)ns + 127) / 128) + (size_t)ns * stage_bytes;
}

// Producer side: acquire stage for the i-th tile (waits for consumers to free it).
__device__ __forceinline__ bool ring_acquire(const Ring& r, int i, int* err) {
  if (i >= r.ns) {
    const int s = i % r.ns;
    return mbar_wait(&r.empty[s], (uint32_t)(((i / r.ns) - 1) & 1), err, kErrTimeoutEmpty);
  }
  return true;
}

// Producer drain: wait (bounded) until the copies of the last issued tiles landed.
__device__ __forceinline__ void ring_drain(const Ring& r, int issued) {
  const int first = issued > r.ns ? issued - r.ns : 0;
  for (int i = first; i < issued; ++i)
    mbar_wait(&r.full[i % r.ns], (uint32_t)((i / r.ns) & 1), nullptr, 0);
}

// --------------------------------------------------------------------------
// Q8_0 GEMV kernel
// --------------------------------------------------------------------------
template <int G, int ORDER, int MODE>
__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv_q8(const __grid_constant__ Q8GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.K / kQBlk;
  const uint32_t rowbytes = (uint32_t)(nb * kQBytes);
  const uint32_t tile_bytes = rowbytes * kTileRows * (MODE == kModeSwiglu ? 2u : 1u);
  const int tiles_per_seg = a.seg_rows / kTileRows;
  const int ntiles = a.nseg * tiles_per_seg;
  // A contiguous run of tiles per CTA: with several segments (layers) in one
  // launch a CTA crosses at most a few segment boundaries, so its x vector is
  // reloaded that often rather than on every tile.
  const int t_begin = (int)((int64_t)blockIdx.x * ntiles / gridDim.x);
  const int t_end = (int)((int64_t)(blockIdx.x + 1) * ntiles / gridDim.x);
  Ring ring = ring_setup(smem, a.nstages, tile_bytes, kGemvConsumerWarps);
  ktrace_start(a.trace);
  // Weights do not depend on the previous kernel: let the next kernel launch
  // and this one's copies start before the previous kernel has finished.
  pdl_launch_dependents();

  if (warp == kGemvConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      // tile t = t_begin + i sits in stage s = i % ns, round i / ns; segment
      // and row are stepped along instead of divided out per tile
      int i = 0, s = 0, seg = t_begin / tiles_per_seg, r0 = (t_begin % tiles_per_seg) * kTileRows;
      uint32_t round_par = 0;
      for (int t = t_begin; t < t_end; ++t, ++i) {
        if (i >= ring.ns && !mbar_wait(&ring.empty[s], round_par ^ 1u, a.err, kErrTimeoutEmpty))
          break;
        const uint8_t* src = a.seg[seg].w + (int64_t)r0 * rowbytes;
        uint8_t* dst = ring.buf + (size_t)s * ring.stage_bytes;
        mbar_expect_tx(&ring.full[s], tile_bytes);
        bulk_g2s(dst, src, rowbytes * kTileRows, &ring.full[s], pol);
        if (MODE == kModeSwiglu)
          bulk_g2s(dst + rowbytes * kTileRows, src + a.up_off_bytes, rowbytes * kTileRows,
                   &ring.full[s], pol);
        if (++s == ring.ns) s = 0, round_par ^= 1u;
        if ((r0 += kTileRows) == a.seg_rows) r0 = 0, ++seg;
      }
      ring_drain(ring, i);
    }
    return;
  }

  // ---------------- consumers ----------------
  __shared__ __align__(16) float xf[G * 32 * kXfStride];
  __shared__ float rs;
  // The decode state (stop, pos, tokens) changes only in a step's last
  // kernel, and gamma never: read them before waiting for the previous kernel.
  const bool stopped = a.seq != nullptr && a.seq->stop != 0;
  constexpr bool kNorm = MODE == kModeNormIn || MODE == kModeSwiglu;
  uint16_t gr[G * 4];
  const uint16_t* xin = a.seg[0].x;
  if (kNorm && !stopped) {
    load_gamma_regs<G * 1024>(a.norm_g, a.K, gr);
    if (a.tokens != nullptr) {
      const int64_t pos = a.seq->pos;
      int64_t tok = 0;
      if (pos < 0 || pos >= a.S) {  // a corrupted state: report it, touch nothing outside
        if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
      } else {
        tok = a.tokens[pos];
        if (tok < 0 || tok >= kVocab) {
          if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadToken);
          tok = 0;
        }
      }
      xin = a.embd + tok * (int64_t)kDim;
    }
  }
  pdl_wait();  // the previous kernel's outputs (activations) are visible
  ktrace_release(a.trace);
  const uint16_t* xcur = nullptr;
  if (kNorm && !stopped) {
    if (a.tokens != nullptr && blockIdx.x == 0 && warp == 0 && a.embed_out != nullptr)
      for (int k = lane; k < a.K; k += 32) a.embed_out[k] = xin[k];
    cta_rmsnorm_to_xf<G * 1024>(xin, gr, a.K, xf, &rs);
  }

  // A warp whose wait timed out keeps walking the tiles without computing,
  // so that every consumer warp still reaches the barriers of an x reload.
  bool live = true;
  int s = 0, seg = t_begin / tiles_per_seg, r0 = (t_begin % tiles_per_seg) * kTileRows;
  uint32_t round_par = 0;
  for (int t = t_begin; t < t_end; ++t) {
    if ((MODE == kModePlain || MODE == kModeResid) && !stopped && a.seg[seg].x != xcur) {
      if (xcur != nullptr) consumer_sync();  // every warp is done with the previous x
      xcur = a.seg[seg].x;
      stage_x_f32(xcur, a.K, xf);
    }
    const int row = r0 + warp;
    uint16_t rres = 0;  // the residual, fetched while the row dot runs
    if (MODE == kModeResid && !stopped && lane == 0) rres = a.seg[seg].r[row];
    live = live && mbar_wait(&ring.full[s], round_par, a.err, kErrTimeoutFull);
    if (live && !stopped) {
      const uint32_t base = smem_u32(ring.buf + (size_t)s * ring.stage_bytes);
      const float d = q8_row_dot_xf<G, ORDER>(base + rowbytes * warp, nb, lane, xf);
      if (MODE == kModeSwiglu) {
        const float u = q8_row_dot_xf<G, ORDER>(base + rowbytes * (kTileRows + warp), nb, lane, xf);
        if (lane == 0) a.seg[seg].y[row] = swiglu_h(f2h(d), f2h(u));
      } else if (MODE == kModeResid) {
        if (lane == 0) a.seg[seg].y[row] = f2h(__fadd_rn(h2f(rres), h2f(f2h(d))));
      } else {
        if (lane == 0) a.seg[seg].y[row] = f2h(d);
      }
    }
    __syncwarp();
    if (live && lane == 0) mbar_arrive(&ring.empty[s]);
    if (++s == ring.ns) s = 0, round_par ^= 1u;
    if ((r0 += kTileRows) == a.seg_rows) r0 = 0, ++seg;
  }
  if (a.advance != nullptr && !stopped && blockIdx.x == 0 && threadIdx.x == 0)
    a.advance->pos += 1;
  ktrace_end(a.trace);
}

// --------------------------------------------------------------------------
// Q8_0 GEMV, one tile per CTA (the batch-1 decode launches)
// --------------------------------------------------------------------------
// Weights do not depend on the previous kernel, so each warp's row (rows:
// gate and up with SwiGLU) lands and is converted to registers -- exact half2
// in the MLIR order, f32 scale * q_j in the CUDA order -- before the wait;
// after it only x (RMSNorm included) and the FMA chains remain.  Same
// operations and orders as k_gemv_q8.
constexpr int kGemv1tThreads = 32 * kTileRows;  // one warp per row of the tile

template <int G, int ORDER>
__device__ __forceinline__ void q8_row_to_regs(uint32_t row, int nb, int lane, float (&q)[G][32],
                                               float (&sc)[G]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int b = lane + 32 * g;
    if (b < nb) {
      const Q8BlockWords bw = q8_load_block(row + (uint32_t)(kQBytes * b));
      sc[g] = h2f((uint16_t)bw.scale16);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float f[4];
        q8x4_to_f32(bw.q[i], f);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          q[g][4 * i + j] = ORDER == kOrderMlir ? f[j] : __fmul_rn(sc[g], f[j]);
      }
    } else {
      sc[g] = 0.0f;
#pragma unroll
      for (int j = 0; j < 32; ++j) q[g][j] = 0.0f;
    }
  }
}

template <int G, int ORDER>
__device__ __forceinline__ float q8_regs_dot_xf(const float (&q)[G][32], const float (&sc)[G],
                                                int nb, int lane, const float* xf) {
  float acc = 0.0f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int b = lane + 32 * g;
    if (b < nb) {
      const float4* xb = reinterpret_cast<const float4*>(xf + b * kXfStride);
      if constexpr (ORDER == kOrderMlir) {
        float inner = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 xv = xb[i];
          inner = __fmaf_rn(q[g][4 * i + 0], xv.x, inner);
          inner = __fmaf_rn(q[g][4 * i + 1], xv.y, inner);
          inner = __fmaf_rn(q[g][4 * i + 2], xv.z, inner);
          inner = __fmaf_rn(q[g][4 * i + 3], xv.w, inner);
        }
        acc = __fmaf_rn(sc[g], inner, acc);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 xv = xb[i];
          acc = __fmaf_rn(q[g][4 * i + 0], xv.x, acc);
          acc = __fmaf_rn(q[g][4 * i + 1], xv.y, acc);
          acc = __fmaf_rn(q[g][4 * i + 2], xv.z, acc);
          acc = __fmaf_rn(q[g][4 * i + 3], xv.w, acc);
        }
      }
    }
  }
  return warp_sum(acc);
}

// The same row kept as exact half2 pairs (16 registers a block instead of 32),
// widened to f32 after the wait: the SwiGLU kernel's up row.
template <int G>
__device__ __forceinline__ void q8_row_to_h2regs(uint32_t row, int nb, int lane,
                                                 uint32_t (&h)[G][16], float (&sc)[G]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int b = lane + 32 * g;
    if (b < nb) {
      const Q8BlockWords bw = q8_load_block(row + (uint32_t)(kQBytes * b));
      sc[g] = h2f((uint16_t)bw.scale16);
#pragma unroll
      for (int i = 0; i < 8; ++i) q8x4_to_h2(bw.q[i], h[g][2 * i], h[g][2 * i + 1]);
    } else {
      sc[g] = 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) h[g][j] = 0u;
    }
  }
}

// Dot of a half2-held row with the f16 copy of x in the MLIR order: the
// inner chain of q_j * x_j (f16 operands, f32 accumulate, one rounding each,
// the same as widening both first), then acc = fma(scale, inner, acc).
template <int G>
__device__ __forceinline__ float q8_h2regs_dot_xh(const uint32_t (&h)[G][16], const float (&sc)[G],
                                                  int nb, int lane, const uint16_t* xh) {
  float acc = 0.0f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int b = lane + 32 * g;
    if (b < nb) {
      const uint4* xb = reinterpret_cast<const uint4*>(xh + b * kXhStride);
      float inner = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 xv = xb[i];
        inner = fma_h2(h[g][4 * i + 0], xv.x, inner);
        inner = fma_h2(h[g][4 * i + 1], xv.y, inner);
        inner = fma_h2(h[g][4 * i + 2], xv.z, inner);
        inner = fma_h2(h[g][4 * i + 3], xv.w, inner);
      }
      acc = __fmaf_rn(sc[g], inner, acc);
    }
  }
  return warp_sum(acc);
}

// Blocks per SM, which caps the registers: 512 QKV tiles need 4 resident,
// 384 gate/up tiles 3; the K = 2048 / 3072 launches (128 tiles) take 3 so
// that the next kernel's CTAs fit beside them (measured: 515 us per traced
// step against 521 with 2 and 529 with 5 / 4 / 3).
template <int G, int MODE>
constexpr int gemv1t_min_blocks() {
  return G > 1 ? 3 : (MODE == kModeSwiglu ? 3 : 4);
}

template <int G, int ORDER, int MODE>
__global__ void __launch_bounds__(kGemv1tThreads, gemv1t_min_blocks<G, MODE>())
    k_gemv_q8_1t(const __grid_constant__ Q8GemvArgs a) {
  static_assert(ORDER == kOrderMlir || MODE != kModeSwiglu, "SwiGLU runs in the MLIR order");
  // Rows are held as exact half2 and multiplied with an f16 copy of x by the
  // mixed-precision FMA: half the registers of f32 rows, so every CTA of a
  // launch, and the next launch's, can be resident before the release, and
  // the f16-operand FMA runs faster here than widening either operand first.
  // The CUDA order (scale * q_j formed first) keeps f32 rows and an f32 x.
  constexpr bool kH2 = ORDER == kOrderMlir;
  constexpr bool kXf = !kH2;
  constexpr bool kXh = kH2 || MODE == kModeSwiglu;
  extern __shared__ __align__(128) uint8_t smem[];  // the tile (gate tile, then up tile)
  __shared__ __align__(8) uint64_t full;
  __shared__ __align__(16) float xf[kXf ? G * 32 * kXfStride : 4];
  __shared__ __align__(16) uint16_t xh[kXh ? G * 32 * kXhStride : 8];
  __shared__ float rs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = a.K / kQBlk;
  const uint32_t rowbytes = (uint32_t)(nb * kQBytes);
  const uint32_t tile_bytes = rowbytes * kTileRows * (MODE == kModeSwiglu ? 2u : 1u);
  const int tiles_per_seg = a.seg_rows / kTileRows;
  const int seg = blockIdx.x / tiles_per_seg;
  const int r0 = (blockIdx.x % tiles_per_seg) * kTileRows;
  ktrace_start(a.trace);
  if (threadIdx.x == 0) {
    mbar_init(&full, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    const uint64_t pol = l2_policy_evict_first();
    const uint8_t* src = a.seg[seg].w + (int64_t)r0 * rowbytes;
    mbar_expect_tx(&full, tile_bytes);
    bulk_g2s(smem, src, rowbytes * kTileRows, &full, pol);
    if (MODE == kModeSwiglu)
      bulk_g2s(smem + rowbytes * kTileRows, src + a.up_off_bytes, rowbytes * kTileRows, &full, pol);
    q8_prefetch_next(a);
  }
  // The decode state (stop, pos, tokens) changes only in a step's last
  // kernel, and gamma never: read them before waiting for the previous kernel.
  const bool stopped = a.seq != nullptr && a.seq->stop != 0;
  constexpr bool kNorm = MODE == kModeNormIn || MODE == kModeSwiglu;
  uint16_t gr[G * 4];
  const uint16_t* xin = a.seg[seg].x;
  if (kNorm && !stopped) {
    load_gamma_regs<G * 1024>(a.norm_g, a.K, gr);
    if (a.tokens != nullptr) {
      const int64_t pos = a.seq->pos;
      int64_t tok = 0;
      if (pos < 0 || pos >= a.S) {  // a corrupted state: report it, touch nothing outside
        if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
      } else {
        tok = a.tokens[pos];
        if (tok < 0 || tok >= kVocab) {
          if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadToken);
          tok = 0;
        }
      }
      xin = a.embd + tok * (int64_t)kDim;
    }
  }
  float q[kH2 ? 1 : G][32], sc[G];
  uint32_t qh[kH2 ? G : 1][16];
  uint32_t qu[MODE == kModeSwiglu ? G : 1][16];
  float scu[MODE == kModeSwiglu ? G : 1];
  const bool landed = mbar_wait_own(&full, 0u, a.err, kErrTimeoutFull);
  if (landed && !stopped) {
    if constexpr (kH2)
      q8_row_to_h2regs<G>(smem_u32(smem) + rowbytes * warp, nb, lane, qh, sc);
    else
      q8_row_to_regs<G, ORDER>(smem_u32(smem) + rowbytes * warp, nb, lane, q, sc);
    if constexpr (MODE == kModeSwiglu)
      q8_row_to_h2regs<G>(smem_u32(smem) + rowbytes * (kTileRows + warp), nb, lane, qu, scu);
  }
  // one decision for the whole CTA: the barriers below need every thread
  const bool work = __syncthreads_and(landed && !stopped) != 0;
  pdl_wait();  // the previous kernel's outputs (activations) are visible
  ktrace_release(a.trace);
  if (work) {
    if (kNorm) {
      if (a.tokens != nullptr && blockIdx.x == 0 && warp == 0 && a.embed_out != nullptr)
        for (int k = lane; k < a.K; k += 32) a.embed_out[k] = xin[k];
      cta_rmsnorm_to_x<G * 1024, kXf, kXh>(xin, gr, a.K, xf, xh, &rs);
    } else {
      stage_x<kXf, kXh>(xin, a.K, xf, xh);
    }
    const int row = r0 + warp;
    uint16_t rres = 0;
    if (MODE == kModeResid && lane == 0) rres = a.seg[seg].r[row];
    float d;
    if constexpr (kH2)
      d = q8_h2regs_dot_xh<G>(qh, sc, nb, lane, xh);
    else
      d = q8_regs_dot_xf<G, ORDER>(q, sc, nb, lane, xf);
    if constexpr (MODE == kModeSwiglu) {
      const float u = q8_h2regs_dot_xh<G>(qu, scu, nb, lane, xh);
      if (lane == 0) a.seg[seg].y[row] = swiglu_h(f2h(d), f2h(u));
    } else if (MODE == kModeResid) {
      if (lane == 0) a.seg[seg].y[row] = f2h(__fadd_rn(h2f(rres), h2f(f2h(d))));
    } else {
      if (lane == 0) a.seg[seg].y[row] = f2h(d);
    }
  }
  if (a.advance != nullptr && !stopped && blockIdx.x == 0 && threadIdx.x == 0)
    a.advance->pos += 1;
  ktrace_end(a.trace);
}

// --------------------------------------------------------------------------
// Residual stream from split projections (the fused engine)
// --------------------------------------------------------------------------
// The fused engine splits the O and down projections along K into kFParts
// f32 partial vectors; a consumer rebuilds the residual stream, 4 elements
// per thread: y = f16(res + f16(((p0 + p1) + p2) + ... + p7)).
constexpr int kFParts = 8;

// f16(res + f16(s)) of 4 elements.
__device__ __forceinline__ uint2 resid_round(uint2 rv, float4 s) {
  auto add = [](uint16_t r, float q) { return f2h(__fadd_rn(h2f(r), h2f(f2h(q)))); };
  uint2 y;
  y.x = (uint32_t)add((uint16_t)(rv.x & 0xffffu), s.x) | ((uint32_t)add((uint16_t)(rv.x >> 16), s.y) << 16);
  y.y = (uint32_t)add((uint16_t)(rv.y & 0xffffu), s.z) | ((uint32_t)add((uint16_t)(rv.y >> 16), s.w) << 16);
  return y;
}

// f16(res + f16(p[0] + ... + p[7])) of 4 elements, the partials summed in order.
__device__ __forceinline__ uint2 resid_finish(uint2 rv, const float4 (&p)[kFParts]) {
  float4 s = p[0];
#pragma unroll
  for (int c = 1; c < kFParts; ++c) {
    s.x = __fadd_rn(s.x, p[c].x);
    s.y = __fadd_rn(s.y, p[c].y);
    s.z = __fadd_rn(s.z, p[c].z);
    s.w = __fadd_rn(s.w, p[c].w);
  }
  return resid_round(rv, s);
}

// resid_finish over partials in shared memory (partial c at p0 + c * stride
// bytes), read one at a time.
__device__ __forceinline__ uint2 resid_finish_smem(uint2 rv, uint32_t p0, uint32_t stride) {
  float4 s;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(s.x), "=f"(s.y), "=f"(s.z), "=f"(s.w)
               : "r"(p0));
#pragma unroll 1
  for (int c = 1; c < kFParts; ++c) {
    float4 t;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(t.x), "=f"(t.y), "=f"(t.z), "=f"(t.w)
                 : "r"(p0 + (uint32_t)c * stride));
    s.x = __fadd_rn(s.x, t.x);
    s.y = __fadd_rn(s.y, t.y);
    s.z = __fadd_rn(s.z, t.z);
    s.w = __fadd_rn(s.w, t.w);
  }
  return resid_round(rv, s);
}

__device__ __forceinline__ uint2 resid_plus_parts(const uint16_t* res, const float* parts, int k0) {
  const uint2 rv = __ldcg(reinterpret_cast<const uint2*>(res + k0));
  float4 p[kFParts];
#pragma unroll
  for (int c = 0; c < kFParts; ++c) p[c] = __ldcg(reinterpret_cast<const float4*>(parts + c * kDim + k0));
  return resid_finish(rv, p);
}

// --------------------------------------------------------------------------
// f16 vocab GEMV + argmax
// --------------------------------------------------------------------------
struct ArgmaxPartial {
  float v;
  int32_t pad;
  int64_t i;
};

// "a is a better argmax candidate than b": larger value, then lower index;
// only values above -inf qualify (NaN never does) -- the strict ogt scan of
// model/qwen3_full.mlir:1482-1507.
__device__ __forceinline__ bool am_better(float av, int64_t ai, float bv, int64_t bi) {
  if (!(av > -__int_as_float(0x7f800000))) return false;
  if (bi < 0) return true;
  return av > bv || (av == bv && ai < bi);
}

struct VocabArgs {
  const uint16_t* w;       // [N, K] f16 rows
  const uint16_t* x;       // input (f16); normalised with norm_g if non-null
  const uint16_t* norm_g;
  // Fused engine (with norm_g): x = f16(xres + f16(sum of the kFParts
  // vectors of xpart)) instead of x.
  const float* xpart;
  const uint16_t* xres;
  uint16_t* logits;        // optional [N] f16
  int N, K;                // N multiple of 8, K == 1024 (lane holds K/32 inputs)
  ArgmaxPartial* partial;  // [gridDim.x]
  unsigned int* counter;   // zero before the first launch; the last CTA re-zeroes it
  int64_t* token_out;      // optional: the argmax
  // Decode-state update done by the last CTA (optional):
  SeqState* seq;           // pos += 1; tokens[pos] = argmax; n_gen / stop bookkeeping
  int64_t* tokens;
  int64_t S;               // positions the token table covers (tokens has S + 1 entries)
  int* err;
  int nstages;
  unsigned long long* trace;  // optional launch timing record (4 values)
};

constexpr int kVocabK = 1024;

__global__ void __launch_bounds__(kGemvThreads) k_vocab_argmax(const __grid_constant__ VocabArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ ArgmaxPartial warp_best[kGemvThreads / 32];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rowbytes = (uint32_t)a.K * 2u;
  const uint32_t tile_bytes = rowbytes * kTileRows;
  const int ntiles = a.N / kTileRows;
  Ring ring = ring_setup(smem, a.nstages, tile_bytes, kGemvConsumerWarps);
  ktrace_start(a.trace);
  pdl_launch_dependents();
  __shared__ __align__(16) uint16_t xs[kVocabK];
  __shared__ float rs;
  __shared__ int stopped_s;

  if (warp == kGemvConsumerWarps) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int i = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
        if (!ring_acquire(ring, i, a.err)) break;
        const int s = i % ring.ns;
        mbar_expect_tx(&ring.full[s], tile_bytes);
        bulk_g2s(ring.buf + (size_t)s * ring.stage_bytes,
                 reinterpret_cast<const uint8_t*>(a.w) + (int64_t)t * tile_bytes, tile_bytes,
                 &ring.full[s], pol);
      }
      ring_drain(ring, i);
    }
  } else {
    // stop changes only in this (the step's last) kernel; gamma never
    const bool stopped = a.seq != nullptr && a.seq->stop != 0;
    uint16_t gr[kVocabK / 256];
    if (a.norm_g != nullptr && !stopped) load_gamma_regs<kVocabK>(a.norm_g, a.K, gr);
    pdl_wait();
    ktrace_release(a.trace);
    if (threadIdx.x == 0) stopped_s = stopped;
    // lane-strided inputs x[l + 32 i], normalised in f32 and rounded to f16
    uint16_t xh[kVocabK / 32];
    if (!stopped) {
      if (a.norm_g != nullptr) {
        if (a.xpart != nullptr)
          *reinterpret_cast<uint2*>(xs + 4 * threadIdx.x) = resid_plus_parts(a.xres, a.xpart, 4 * threadIdx.x);
        cta_rmsnorm_to_smem_g<kVocabK>(a.xpart != nullptr ? nullptr : a.x, gr, a.K, xs, &rs);
#pragma unroll
        for (int i = 0; i < kVocabK / 32; ++i) xh[i] = xs[lane + 32 * i];
      } else {
#pragma unroll
        for (int i = 0; i < kVocabK / 32; ++i) xh[i] = a.x[lane + 32 * i];
      }
    }
    float best_v = -__int_as_float(0x7f800000);
    int64_t best_i = -1;
    int i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int s = i % ring.ns;
      if (!mbar_wait(&ring.full[s], (uint32_t)((i / ring.ns) & 1), a.err, kErrTimeoutFull)) break;
      if (stopped) {  // drain the ring without computing
        __syncwarp();
        if (lane == 0) mbar_arrive(&ring.empty[s]);
        continue;
      }
      const uint32_t row = smem_u32(ring.buf + (size_t)s * ring.stage_bytes) + rowbytes * warp;
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k < kVocabK / 32; ++k) acc = fma_h(lds16(row + 2u * (lane + 32 * k)), xh[k], acc);
      acc = warp_sum(acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&ring.empty[s]);
      const uint16_t lh = f2h(acc);
      const int64_t n = (int64_t)t * kTileRows + warp;
      if (lane == 0 && a.logits != nullptr) a.logits[n] = lh;
      const float lv = h2f(lh);
      if (am_better(lv, n, best_v, best_i)) {
        best_v = lv;
        best_i = n;
      }
    }
    if (lane == 0) {
      warp_best[warp].v = best_v;
      warp_best[warp].i = best_i;
    }
  }
  __syncthreads();
  if (stopped_s) return;
  if (threadIdx.x == 0) {
    float bv = -__int_as_float(0x7f800000);
    int64_t bi = -1;
    for (int w = 0; w < kGemvConsumerWarps; ++w)
      if (am_better(warp_best[w].v, warp_best[w].i, bv, bi)) {
        bv = warp_best[w].v;
        bi = warp_best[w].i;
      }
    a.partial[blockIdx.x].v = bv;
    a.partial[blockIdx.x].i = bi;
    __threadfence();
    const unsigned prev = atomicAdd(a.counter, 1u);
    is_last = (prev == gridDim.x - 1);
  }
  __syncthreads();
  ktrace_end(a.trace);
  if (!is_last) return;
  __threadfence();
  // the decode state, loaded by thread 0 now (its loads in flight with the
  // partials'; only this thread changes it during the launch)
  int64_t s_pos = 0, s_prompt = 0, s_gen = 0, s_max = 0, s_eos = 0;
  if (threadIdx.x == 0 && a.seq != nullptr) {
    const volatile SeqState* vs = a.seq;
    s_pos = vs->pos;
    s_prompt = vs->n_prompt;
    s_gen = vs->n_gen;
    s_max = vs->max_gen;
    s_eos = vs->eos;
  }
  // last CTA: reduce the per-CTA partials (any order: the rule is a total
  // order); a thread's two partials are loaded before either is compared
  float bv = -__int_as_float(0x7f800000);
  int64_t bi = -1;
  const int nc = (int)gridDim.x, nt = (int)blockDim.x;
  for (int c = threadIdx.x; c < nc; c += 2 * nt) {
    const volatile ArgmaxPartial* p = a.partial + c;
    const float v = p->v;
    const int64_t ii = p->i;
    const bool two = c + nt < nc;
    float v2 = -__int_as_float(0x7f800000);
    int64_t i2 = -1;
    if (two) {
      v2 = p[nt].v;
      i2 = p[nt].i;
    }
    if (am_better(v, ii, bv, bi)) {
      bv = v;
      bi = ii;
    }
    if (two && am_better(v2, i2, bv, bi)) {
      bv = v2;
      bi = i2;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (am_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    warp_best[warp].v = bv;
    warp_best[warp].i = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
      if (am_better(warp_best[w].v, warp_best[w].i, bv, bi)) {
        bv = warp_best[w].v;
        bi = warp_best[w].i;
      }
    if (a.token_out != nullptr) *a.token_out = bi;
    if (a.seq != nullptr) {
      SeqState* st = a.seq;
      const int64_t pos = s_pos;
      if (pos < 0 || pos >= a.S) {  // a corrupted state: report it, write nothing
        if (a.err) atomicCAS(a.err, 0, kErrBadPos);
        st->stop = 1;
        *a.counter = 0u;
        return;
      }
      a.tokens[pos + 1] = bi;
      if (pos >= s_prompt) {
        const int64_t n_gen = s_gen + 1;
        st->n_gen = n_gen;
        // @generate (model/qwen3_full.mlir:1412-1530): groups of 4; the loop
        // ends when the last token of a group is eos, or max_gen is reached.
        if (n_gen >= s_max || ((n_gen % 4) == 0 && bi == s_eos)) st->stop = 1;
      }
      st->pos = pos + 1;
    }
    *a.counter = 0u;
  }
  ktrace_end(a.trace);
}

}  // namespace q3
