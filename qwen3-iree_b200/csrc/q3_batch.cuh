// q3_batch.cuh -- batched decode (B independent sequences, B <= 64) for sm_100a.
//
// At batch 16-64 a projection is a real contraction, [B,K] x [K,N], and runs
// on the 5th-generation tensor cores: tcgen05.mma (kind::f16, M=128 weight
// rows, N = B padded to a multiple of 16, f32 accumulators in TMEM).
//
// Q8_0 weights (k_bgemm_q8): a producer thread brings 128 rows x 256 K of raw
// Q8_0 bytes into shared memory with one tensor TMA (the row stride of the
// reference layout is a multiple of 16 bytes, so a [128 x 272-byte] box
// works) and the activations' K-slices with SWIZZLE_128B tensor TMA; eight
// dequantising warps turn each 64-wide K-slice into f16 weights in the
// canonical SWIZZLE_128B layout -- w = f16(scale * q), the f16 dequant of the
// reference's own fused-GEMV region (model/qwen3_full.mlir:564-579) -- and one
// thread issues the MMAs.  The same warps read the accumulators back with
// tcgen05.ld (four of them for a single-CTA tile, all eight for a split tile's
// partial) and apply the epilogue (residual add, or SwiGLU over a gate tile
// and its up tile held in two accumulators).
//
// f16 vocab head (k_bvocab): weight tiles and activations both arrive by
// SWIZZLE_128B tensor TMA; each CTA walks tiles of 128 vocabulary rows,
// rounds logits to f16 and keeps, per sequence, the first index of the
// largest value; the last CTA reduces the per-CTA candidates and advances the
// sequences.
//
// Accumulation order inside the tensor core is not the reference kernels'
// order, so batched results agree with the CPU oracle within a tolerance
// (rel-L2 <= 1e-3), not bit for bit; the batch-1 path is the bit-exact one.
#pragma once

#include "q3_attn.cuh"
#include "q3_common.cuh"
#include "q3_gemv.cuh"
#include "q3_tc.cuh"

namespace q3 {

constexpr int kBMaxBatch = 64;
constexpr int kBgDqWarps = 8;                     // dequantising warps (one Q8_0 block each)
constexpr int kBgThreads = 64 + 32 * kBgDqWarps;  // warp 0 TMA, warp 1 MMA, warps 2-9 dequant
constexpr int kBvThreads = 192;                   // vocab: warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kBgSubStages = 4;
constexpr uint32_t kBgRawBytes = 128u * 272u;  // 128 rows x 8 Q8_0 blocks
constexpr uint32_t kBgAtomA = 128u * 128u;     // 128 rows x 64 f16, SWIZZLE_128B

enum BGemmMode : int { kBgPlain = 0, kBgResid = 1, kBgSwiglu = 2 };

// A pipeline wait of the batched kernels gives up after ~1 s of SM clock
// (kSpinCycles, as every other wait here; a decode step takes milliseconds)
// and records in the error word
//   bits 0-3: kErrTimeout*, bits 4-7: wait site, bits 8-15: launch tag
//   (layer * 8 + kernel), bits 16-27: CTA index.
constexpr long long kBatchSpinCycles = kSpinCycles;
__device__ __forceinline__ int bwait_code(int code, int site, int tag) {
  return code | (site << 4) | ((tag & 0xff) << 8) | (((int)blockIdx.x & 0xfff) << 16);
}
// Per-CTA phase stamps (global timer, ns) of the batched kernels' traced
// launches: p[cta * kBPhases + k], written by one chosen thread.
constexpr int kBPhases = 8;
__device__ __forceinline__ void bphase(long long* p, int k, bool me) {
  if (p != nullptr && me) {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    p[(int64_t)(blockIdx.y * gridDim.x + blockIdx.x) * kBPhases + k] = t;
  }
}

#define Q3_BWAIT(bar, parity, code, site) \
  mbar_wait_own((bar), (parity), a.err, bwait_code((code), (site), a.tag), kBatchSpinCycles)

// Device state of one sequence of a batch.
struct BatchSeq {
  int64_t pos;       // position of the token fed this step
  int64_t n_gen;     // tokens generated so far
  int64_t n_prompt;  // tokens[pos+1] is overwritten only once pos+1 >= n_prompt
  int64_t pad;
};

struct BGemmArgs {
  CUtensorMap wmap[3];   // Q8_0 weights viewed as u16 [rows_total, rowbytes/2], box {136, 128}
  CUtensorMap xmap;      // activations f16 [npad, K], box {64, npad}, SWIZZLE_128B
  int wseg_rows[3];      // output rows served by wmap[i] (segments concatenated)
  int64_t wrow0[3];      // first weight row (layer * N) in each map
  int K;
  int kc;                // 256-wide K chunks per CTA (1 or 2); gridDim.y = K / 256 / kc
  int B;                 // live sequences (<= npad)
  int ldy;               // output row stride (elements) per sequence
  uint16_t* y;           // [npad][ldy] f16
  const uint16_t* r;     // residual [npad][ldy] (kBgResid)
  int64_t up_rows;       // kBgSwiglu: offset (rows) from a gate row to its up row
  int* err;              // optional device error word (pipeline wait timed out)
  int tag;               // launch tag recorded with a timeout
  unsigned long long* trace;  // optional launch timing record
  long long* phase;      // optional per-CTA phase stamps [CTAs][kBPhases] (ns)
  // RMSNorm folded into the projections (model/qwen3_full.mlir:134-165),
  // y = W (x / r_b * gamma) computed as (W f16(x * gamma)) / r_b.  A
  // residual-producing launch (kBgResid, split) writes, per reducing CTA,
  // the sum of squares of its f16 outputs of each row b,
  // ssq_out[(tile * splits + rank) * 64 + b] (whole 128-row blocks per CTA),
  // and the next projection's operand xg_out = f16(out * xg_gamma).  A
  // normalising launch (its xmap over that operand) multiplies each reduced
  // sum by 1 / r_b, r_b = sqrt(sum_p ssq_in[p * 64 + b] / K + eps) over
  // p < ssq_parts in p order, before the epilogue.
  float* ssq_out;
  uint16_t* xg_out;       // [npad][ldy]
  const uint16_t* xg_gamma;
  const float* ssq_in;
  int ssq_parts;
};

// Weight stages (dequantised 64-wide K slices) between the dequantising warps
// and the MMA thread; two accumulators (gate + up) leave room for two.
__host__ __device__ constexpr int bgemm_substages(int naccum) { return naccum == 2 ? 2 : 4; }
constexpr int kBgMaxKc = 2;       // chunks per CTA: all of its activations stay resident
constexpr int kBgMaxSplits = 8;   // CTAs per tile = one portable cluster

// Items of the split reduction per CTA: ceil(total / splits), rounded up to
// whole 128-row blocks (item = b*128 + row: a CTA reduces whole rows b).
__host__ __device__ constexpr int bgemm_red_per(int total, int splits) {
  return ((total + splits - 1) / splits + 127) / 128 * 128;
}

// Dynamic shared memory: weight stages (reused for the f32 partials), every
// activation slice of the CTA's K range, and one raw stage per chunk.
__host__ __device__ constexpr size_t bgemm_smem_bytes(int npad, int naccum, int kc) {
  return 1024 /*align slack*/ + (size_t)naccum * bgemm_substages(naccum) * kBgAtomA +
         (size_t)kc * 4 * npad * 128 + (size_t)kc * naccum * kBgRawBytes;
}

__device__ __forceinline__ void lds128(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c,
                                       uint32_t& d) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}

// Dequantise Q8_0 block BLK (0/1) of 64-wide slice J of weight row r into
// chunks 4*BLK .. 4*BLK+3 of row r of the SWIZZLE_128B atom, as f16(scale*q)
// (model/qwen3_full.mlir:564-579).  The block's 34 bytes sit at stage offset
// r*272 + 68J + 34BLK; three 16-byte loads from the 16-byte boundary D bytes
// below cover them, and with rows 272 = 17*16 bytes apart the 8 rows of a
// quarter warp fall on distinct bank groups.
template <int J, int BLK>
__device__ __forceinline__ void dequant_block(uint32_t stage, uint32_t atom, uint32_t r) {
  constexpr int D = (4 * J + 2 * BLK) & 15;
  const uint32_t a0 = stage + r * 272u + (uint32_t)(68 * J + 34 * BLK - D);
  uint32_t w[12];
  lds128(a0, w[0], w[1], w[2], w[3]);
  lds128(a0 + 16, w[4], w[5], w[6], w[7]);
  lds128(a0 + 32, w[8], w[9], w[10], w[11]);
  const uint32_t sc = (D & 2) ? (w[D >> 2] >> 16) : (w[D >> 2] & 0xffffu);
  const uint32_t s2 = sc | (sc << 16);
  constexpr int Q = (D + 2) >> 2;  // word holding the first q byte
  uint32_t q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    q[i] = ((D + 2) & 3) == 0 ? w[Q + i] : __byte_perm(w[Q + i], w[Q + i + 1], 0x5432);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t a01, a23, b01, b23;
    q8x4_to_h2(q[2 * c], a01, a23);
    q8x4_to_h2(q[2 * c + 1], b01, b23);
    uint32_t o0, o1, o2, o3;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o0) : "r"(a01), "r"(s2));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o1) : "r"(a23), "r"(s2));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o2) : "r"(b01), "r"(s2));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o3) : "r"(b23), "r"(s2));
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                     atom + sw128_chunk_offset(r, (uint32_t)(4 * BLK + c))),
                 "r"(o0), "r"(o1), "r"(o2), "r"(o3)
                 : "memory");
  }
}

template <int J>
__device__ __forceinline__ void dequant_block_j(int blk, uint32_t stage, uint32_t atom, uint32_t r) {
  if (blk == 0)
    dequant_block<J, 0>(stage, atom, r);
  else
    dequant_block<J, 1>(stage, atom, r);
}


// Batched Q8_0 GEMM.  Grid (row tiles, S splits), clusters of the S CTAs of
// a tile: CTA (t, s) owns output rows 128t .. 128t+127 (kBgSwiglu: those gate
// rows and their up rows) over 256-wide K chunks [s*kc, (s+1)*kc).  With
// S = 1 the CTA applies the epilogue straight from TMEM.  With S > 1 each CTA
// leaves its f32 partial in its own shared memory; after a cluster barrier
// CTA s reduces items [s*n/S, (s+1)*n/S) of the tile's 128 x NPAD outputs,
// reading the S partials over distributed shared memory in split order (the
// same bits whatever the timing), and applies the epilogue.  Every activation
// slice of the CTA's K range is loaded once, and the weight copies and their
// dequantisation start before the wait on the previous kernel (weights do
// not depend on it).  NPAD = batch padded to 16.
template <int NPAD, int MODE>
__global__ void __launch_bounds__(kBgThreads, 1) k_bgemm_q8(const __grid_constant__ BGemmArgs a) {
  constexpr int NACC = MODE == kBgSwiglu ? 2 : 1;   // accumulators (gate, up)
  constexpr int SUB = bgemm_substages(NACC);
  constexpr uint32_t TCOLS = NPAD * NACC <= 32 ? 32 : NPAD * NACC <= 64 ? 64 : 128;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t raw_full[kBgMaxKc], x_full, acc_full, red_bar;
  __shared__ __align__(8) uint64_t a_full[kBgSubStages], a_empty[kBgSubStages];
  __shared__ uint32_t tmem_base;
  __shared__ float red_ss[2 * NPAD];         // per-warp sums of squares of the outputs
  constexpr int kRPre = 8;                   // residuals of a thread staged before the shares
  __shared__ uint16_t rstage[MODE == kBgResid ? kRPre * 256 : 1];
  __shared__ float rs_b[kBMaxBatch];         // 1 / RMS of the rows (folded norm)
  __shared__ float rs_g[2][kBMaxBatch];      // their partial sums of squares
  const bool fold = a.ssq_in != nullptr;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunk = a.kc;
  const int nsub = nchunk * 4;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sA = base;                                // [NACC][SUB][16 KB]; partials later
  const uint32_t sX = sA + NACC * SUB * kBgAtomA;          // [nsub][NPAD*128]
  const uint32_t sR = sX + nsub * NPAD * 128;              // [nchunk][NACC][34816]
  uint8_t* const gbase = smem_raw + (base - smem_u32(smem_raw));
  const int splits = (int)gridDim.y;
  const int cbase = (int)blockIdx.y * nchunk;              // first 256-wide chunk of this CTA
  const int tile = blockIdx.x, n0 = tile * 128;
  ktrace_start(a.trace);
  bphase(a.phase, 0, threadIdx.x == 0);  // start

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBgMaxKc; ++i) mbar_init(&raw_full[i], 1);
    for (int i = 0; i < SUB; ++i) {
      mbar_init(&a_full[i], kBgDqWarps);
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(&x_full, 1);
    mbar_init(&acc_full, 1);
    mbar_init(&red_bar, 1);
    fence_mbar_init();
    if (gridDim.y > 1) {  // the bytes of this CTA's share of the split reduction
      const int total = 128 * NPAD, per = bgemm_red_per(total, (int)gridDim.y);
      const int i0 = (int)cluster_rank() * per;
      const int len = i0 >= total ? 0 : (total - i0 < per ? total - i0 : per);
      mbar_expect_tx(&red_bar, (uint32_t)((int)gridDim.y * NACC * len * 4));
    }
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tmem = tmem_base;
  const uint32_t idesc = idesc_f16_f32(128, NPAD);

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      // which weight map serves rows n0.. (segments concatenated)
      int seg = 0;
      int64_t row = n0;
      while (seg < 2 && row >= a.wseg_rows[seg]) {
        row -= a.wseg_rows[seg];
        ++seg;
      }
      const CUtensorMap* wm = &a.wmap[seg];
      const int y0 = (int)(a.wrow0[seg] + row);
      prefetch_tmap(wm);
      prefetch_tmap(&a.xmap);
      // weights do not depend on the previous kernel: start them first
      for (int c = 0; c < nchunk; ++c) {
        mbar_expect_tx(&raw_full[c], NACC * kBgRawBytes);
        for (int acc = 0; acc < NACC; ++acc)
          tma_load_2d(gbase + (sR - base) + (c * NACC + acc) * kBgRawBytes, wm, (cbase + c) * 136,
                      y0 + (int)(acc * a.up_rows), &raw_full[c]);
      }
      pdl_wait();  // activations come from the previous kernel
      ktrace_release(a.trace);
      bphase(a.phase, 1, true);  // release
      mbar_expect_tx(&x_full, (uint32_t)(nsub * NPAD * 128));
      for (int i = 0; i < nsub; ++i)
        tma_load_2d(gbase + (sX - base) + i * NPAD * 128, &a.xmap, (cbase * 4 + i) * 64, 0, &x_full);
      // the CTA may not exit before every copy has landed
      for (int c = 0; c < nchunk; ++c) Q3_BWAIT(&raw_full[c], 0, kErrTimeoutFull, 3);
      bphase(a.phase, 2, true);  // weights landed (stamped after the release)
      Q3_BWAIT(&x_full, 0, kErrTimeoutFull, 4);
      bphase(a.phase, 3, true);  // activations landed
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = Q3_BWAIT(&x_full, 0, kErrTimeoutFull, 6);
      for (int i = 0; ok && i < nsub; ++i) {
        const int ss = i % SUB;
        if (!Q3_BWAIT(&a_full[ss], (i / SUB) & 1, kErrTimeoutFull, 5)) break;
        tc_fence_after();
        for (int acc = 0; acc < NACC; ++acc) {
          const uint32_t aa = sA + (acc * SUB + ss) * kBgAtomA;
          const uint32_t xx = sX + i * NPAD * 128;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + acc * NPAD, sw128_desc(aa + 32 * kk), sw128_desc(xx + 32 * kk), idesc,
                     (i | kk) != 0);
        }
        umma_commit(&a_empty[ss]);
      }
      umma_commit(&acc_full);
      Q3_BWAIT(&acc_full, 0, kErrTimeoutFull, 7);  // no MMA in flight at dealloc
    }
  } else {
    // ------------------------------------------------ dequant (8 warps)
    const uint32_t r = 32u * (uint32_t)(warp & 3) + lane;  // weight row = TMEM lane
    const int blk = (warp - 2) >> 2;                       // Q8_0 block of each 64-wide slice
    for (int c = 0; c < nchunk; ++c) {
      if (!Q3_BWAIT(&raw_full[c], 0, kErrTimeoutFull, 8)) break;
      bool ok = true;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = c * 4 + j, ss = i % SUB;
        if (i >= SUB && !Q3_BWAIT(&a_empty[ss], ((i / SUB) - 1) & 1, kErrTimeoutEmpty, 9)) {
          ok = false;
          break;
        }
        for (int acc = 0; acc < NACC; ++acc) {
          const uint32_t stage = sR + (c * NACC + acc) * kBgRawBytes;
          const uint32_t atom = sA + (acc * SUB + ss) * kBgAtomA;
          if (j == 0) dequant_block_j<0>(blk, stage, atom, r);
          if (j == 1) dequant_block_j<1>(blk, stage, atom, r);
          if (j == 2) dequant_block_j<2>(blk, stage, atom, r);
          if (j == 3) dequant_block_j<3>(blk, stage, atom, r);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[ss]);
      }
      if (!ok) break;
    }
    if (fold && warp >= 6) {
      // 1 / r_b of every row, by the warps the accumulators do not need, while
      // the MMAs run: row b's parts by 2 threads (32 loads issued together
      // each), the two sums in order; read after the cluster barrier
      pdl_wait();  // the parts come from the previous kernel
      const int t = threadIdx.x - 192, b = t & 63, grp = t >> 6;
      float v[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int q = grp * 32 + u;
        v[u] = (b < NPAD && q < a.ssq_parts) ? __ldcg(a.ssq_in + q * 64 + b) : 0.0f;
      }
      float t32 = v[0];
#pragma unroll
      for (int u = 1; u < 32; ++u) t32 = __fadd_rn(t32, v[u]);
      rs_g[grp][b] = t32;
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (t < kBMaxBatch)
        rs_b[t] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(__fadd_rn(rs_g[0][t], rs_g[1][t]), (float)a.K), kEps)));
    }
    // ------------------------------------------------ accumulators out of TMEM
    // (warps 2-5 for the direct epilogue; with splits all 8 dequant warps:
    // warp w reads TMEM lanes 32*(w%4).. of every 16-column group, warps 2-5
    // the even groups and warps 6-9 the odd ones)
    if (warp < 6 || splits > 1) {
      const bool have = Q3_BWAIT(&acc_full, 0, kErrTimeoutFull, 10);
      bphase(a.phase, 4, threadIdx.x == 64);  // accumulators complete
      tc_fence_after();
      const uint32_t lane_base = (32u * (uint32_t)(warp & 3)) << 16;
      if (have && splits == 1) {
        pdl_wait();  // reads the residual stream / writes buffers of earlier kernels
        const int n = n0 + (int)r;
#pragma unroll
        for (int col0 = 0; col0 < NPAD; col0 += 16) {
          uint32_t v[16], u[16];
          tmem_ld16(tmem + lane_base + col0, v);
          if (MODE == kBgSwiglu) tmem_ld16(tmem + lane_base + NPAD + col0, u);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int b = col0 + j;
            if (b < a.B) {
              const float g = __uint_as_float(v[j]);
              uint16_t out;
              if (MODE == kBgSwiglu)
                out = swiglu_h(f2h(g), f2h(__uint_as_float(u[j])));
              else if (MODE == kBgResid)
                out = f2h(__fadd_rn(h2f(a.r[(int64_t)b * a.ldy + n]), h2f(f2h(g))));
              else
                out = f2h(g);
              a.y[(int64_t)b * a.ldy + n] = out;
            }
          }
        }
      } else if (splits > 1) {
        // partial [acc][b][row] f32 over the (now idle) raw weight stages:
        // group g = TMEM columns 16g.. = (acc, b) columns acc*NPAD + 16g'..;
        // this warp's groups are all loaded before one wait
        constexpr int NG = NACC * NPAD / 16, NGH = (NG + 1) / 2;
        const int half = (warp - 2) >> 2;
        uint32_t v[NGH][16];
        const bool all = __all_sync(0xffffffffu, have);  // TMEM loads are warp-wide
#pragma unroll
        for (int k = 0; k < NGH; ++k) {
          if (2 * k + half >= NG) continue;
          if (all) {
            tmem_ld16(tmem + lane_base + (uint32_t)((2 * k + half) * 16), v[k]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[k][j] = 0u;
          }
        }
        if (all) tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < NGH; ++k) {
          const int g = 2 * k + half;
          if (g < NG) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              asm volatile("st.shared.b32 [%0], %1;" ::"r"(sR + (uint32_t)(((g * 16 + j) * 128 + (int)r) * 4)),
                           "r"(v[k][j])
                           : "memory");
          }
        }
      }
    }
  }
  if (splits > 1) {
    // ------------------------------------------------ cluster reduction
    // CTA d reduces items [d*per, (d+1)*per) of the tile's 128 x NPAD outputs
    // (item = b*128 + row).  After one cluster barrier (every CTA's MMAs are
    // done, so every weight-stage region is free), each CTA pushes its
    // partial of those items into CTA d's stage region as R[s][acc][j] with
    // 16-byte st.async whose bytes count on d's red_bar; d waits for its
    // bytes and sums R[0..S-1] in split order (the same bits whatever the
    // timing).  No CTA touches another's shared memory after its own wait.
    __syncwarp();
    cluster_sync_all();
    bphase(a.phase, 5, threadIdx.x == 64);  // every split's partial stored
    const int total = 128 * NPAD, per = bgemm_red_per(total, splits);
    const int me = (int)cluster_rank();
    if (warp >= 2) {
      const int t = threadIdx.x - 64;  // 0 .. 255
      for (int dst = 0; dst < splits; ++dst) {
        const int i0 = dst * per;
        const int len = i0 >= total ? 0 : (total - i0 < per ? total - i0 : per);
        for (int acc = 0; acc < NACC; ++acc)
          for (int j4 = t; j4 < len / 4; j4 += 2 * 32 * kBgDqWarps) {  // two loads, then two pushes
            const bool two = j4 + 32 * kBgDqWarps < len / 4;
            uint4 v, w;
            lds128(sR + (uint32_t)(((acc * total) + i0 + 4 * j4) * 4), v.x, v.y, v.z, v.w);
            if (two)
              lds128(sR + (uint32_t)(((acc * total) + i0 + 4 * (j4 + 32 * kBgDqWarps)) * 4), w.x, w.y, w.z, w.w);
            st_async_v4(sA + (uint32_t)(((me * NACC + acc) * per + 4 * j4) * 4), (uint32_t)dst, v,
                        smem_u32(&red_bar));
            if (two)
              st_async_v4(sA + (uint32_t)(((me * NACC + acc) * per + 4 * (j4 + 32 * kBgDqWarps)) * 4),
                          (uint32_t)dst, w, smem_u32(&red_bar));
          }
      }
      pdl_wait();  // reads the residual stream / writes buffers of earlier kernels
      const int i0 = me * per;
      const int i1 = i0 + per < total ? i0 + per : total;
      // every item i0 + 256 jj + t of thread t lies in output row n (i0 and
      // the 256-item stride are whole 128-row blocks)
      const int n = n0 + (t & 127);
      if (MODE == kBgResid) {
        // the residuals of this thread's first kRPre items: the loads in
        // flight together while the shares travel, kept for this thread
        uint16_t rv[kRPre];
#pragma unroll
        for (int jj = 0; jj < kRPre; ++jj) {
          const int i = i0 + jj * 256 + t;
          rv[jj] = (i < i1 && (i >> 7) < a.B) ? a.r[(int64_t)(i >> 7) * a.ldy + n] : (uint16_t)0;
        }
#pragma unroll
        for (int jj = 0; jj < kRPre; ++jj) rstage[jj * 256 + t] = rv[jj];
      }
      const bool got = Q3_BWAIT(&red_bar, 0, kErrTimeoutFull, 11);
      bphase(a.phase, 6, threadIdx.x == 64);  // this CTA's shares arrived
      const bool want_ss = MODE == kBgResid && a.ssq_out != nullptr;
      const float gam = MODE == kBgResid && a.xg_out != nullptr ? h2f(a.xg_gamma[n]) : 0.0f;
      for (int jj = 0; i0 + jj * 256 < i1; ++jj) {  // uniform over the 256 threads
        const int i = i0 + jj * 256 + t;
        const int b = i >> 7;
        float sq = 0.0f;
        if (got && i < i1 && b < a.B) {
          float sum[NACC];
#pragma unroll
          for (int acc = 0; acc < NACC; ++acc) {
            // the shares' loads issued together, then summed in split order
            float v[kBgMaxSplits];
#pragma unroll
            for (int sp = 0; sp < kBgMaxSplits; ++sp) {
              if (sp < splits)
                asm volatile("ld.shared.f32 %0, [%1];"
                             : "=f"(v[sp])
                             : "r"(sA + (uint32_t)(((sp * NACC + acc) * per + (i - i0)) * 4)));
            }
            float s0 = v[0];
#pragma unroll
            for (int sp = 1; sp < kBgMaxSplits; ++sp)
              if (sp < splits) s0 = __fadd_rn(s0, v[sp]);
            sum[acc] = fold ? __fmul_rn(s0, rs_b[b]) : s0;
          }
          uint16_t out;
          if (MODE == kBgSwiglu)
            out = swiglu_h(f2h(sum[0]), f2h(sum[NACC - 1]));
          else if (MODE == kBgResid)
            out = f2h(__fadd_rn(h2f(jj < kRPre ? rstage[jj * 256 + t] : a.r[(int64_t)b * a.ldy + n]),
                                h2f(f2h(sum[0]))));
          else
            out = f2h(sum[0]);
          a.y[(int64_t)b * a.ldy + n] = out;
          const float ov = h2f(out);
          sq = __fmul_rn(ov, ov);
          if (MODE == kBgResid && a.xg_out != nullptr)
            a.xg_out[(int64_t)b * a.ldy + n] = f2h(__fmul_rn(ov, gam));
        }
        if (want_ss) {  // a warp's 32 items lie in one row b
          sq = warp_sum(sq);
          if ((t & 31) == 0) red_ss[jj * 8 + (t >> 5)] = sq;
        }
      }
      if (want_ss) {
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (t < kBMaxBatch) {
          float s4 = 0.0f;
          if (t * 128 >= i0 && t * 128 < i1) {  // row t's 4 warp sums, in order
            const int w0 = (t * 128 - i0) >> 5;
            s4 = __fadd_rn(__fadd_rn(red_ss[w0], red_ss[w0 + 1]), __fadd_rn(red_ss[w0 + 2], red_ss[w0 + 3]));
          }
          a.ssq_out[((int64_t)tile * splits + me) * 64 + t] = s4;
        }
      }
      if (!got) Q3_BWAIT(&red_bar, 0, kErrTimeoutFull, 12);  // pushes into this CTA landed
    }
  }
  // role branches and per-lane polling leave warps diverged: reconverge each
  // warp before the CTA barrier (bar.sync counts a warp when its first
  // threads arrive)
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  // The end stamps come from warp 1 after it frees TMEM: per-CTA stamps show
  // warp 1 leaving this barrier only after the epilogue warps reach it, but
  // thread 0 leaving it 1.5-7 us before them (warp 0 has nothing left to do)
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TCOLS);
  }
  bphase(a.phase, 7, threadIdx.x == 32);  // end
  ktrace_end(a.trace, 32);
}

// Per-sequence RMSNorm of model/qwen3_full.mlir:134-165 into the GEMM operand
// buffer xn [npad][K] (padding rows stay zero).  With `tokens`, the input of
// sequence b is embedding row tokens[b * tok_stride + seq[b].pos] and is also
// stored as the residual stream x; with ssq_out the kernel writes each row's
// sum of squares ssq_out[b] and xn = f16(x * gamma) instead, the operand of a
// projection that folds the 1 / r_b in (k_bgemm_q8's ssq_in).
struct BNormArgs {
  const uint16_t* x;     // [npad][K] residual (ignored when tokens != nullptr)
  uint16_t* x_out;       // embedding copy target (tokens != nullptr)
  const uint16_t* gamma;
  uint16_t* xn;          // [npad][K]
  int K;
  int B;
  const int64_t* tokens; // row b's token at position p: tokens[b * tok_stride + p]
  int64_t tok_stride;    // 0 when every row reads one sequence's tokens
  int64_t tok_len;       // positions per row
  const BatchSeq* seq;
  const uint16_t* embd;
  float* ssq_out;        // [64]: sum of squares of each row (rows >= B: 0)
  int* err;
  unsigned long long* trace;  // optional launch timing record
};

__global__ void __launch_bounds__(256) k_bnorm(const __grid_constant__ BNormArgs a) {
  __shared__ __align__(16) uint16_t xs[3072];
  __shared__ float rs;
  const int b = blockIdx.x;
  ktrace_start(a.trace);
  pdl_launch_dependents();
  pdl_wait();
  ktrace_release(a.trace);
  if (b >= a.B) return;
  const uint16_t* x = a.x + (int64_t)b * a.K;
  if (a.tokens != nullptr) {
    const int64_t pos = a.seq[b].pos;
    int64_t tok = 0;
    if (pos < 0 || pos >= a.tok_len) {
      if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    } else {
      tok = a.tokens[(int64_t)b * a.tok_stride + pos];
      if (tok < 0 || tok >= kVocab) {
        if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadToken);
        tok = 0;
      }
    }
    x = a.embd + tok * (int64_t)kDim;
    for (int i = threadIdx.x; i < a.K / 8; i += 256)
      reinterpret_cast<uint4*>(a.x_out + (int64_t)b * a.K)[i] = reinterpret_cast<const uint4*>(x)[i];
  }
  if (a.ssq_out != nullptr) {
    // the row's sum of squares (threads' strided partials, then the 8 warps in order)
    __shared__ float wss[8];
    float ss = 0.0f;
    for (int k = threadIdx.x; k < a.K; k += 256) {
      const float v = h2f(x[k]);
      ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) wss[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = wss[0];
      for (int w = 1; w < 8; ++w) t = __fadd_rn(t, wss[w]);
      a.ssq_out[b] = t;
    }
    if (b == 0)
      for (int r = a.B + (int)threadIdx.x; r < kBMaxBatch; r += 256) a.ssq_out[r] = 0.0f;
  }
  if (a.ssq_out != nullptr) {
    for (int k = threadIdx.x; k < a.K; k += 256)
      a.xn[(int64_t)b * a.K + k] = f2h(__fmul_rn(h2f(x[k]), h2f(a.gamma[k])));
  } else {
    cta_rmsnorm_to_smem(x, a.gamma, a.K, xs, &rs);
    for (int i = threadIdx.x; i < a.K / 8; i += 256)
      reinterpret_cast<uint4*>(a.xn + (int64_t)b * a.K)[i] = reinterpret_cast<const uint4*>(xs)[i];
  }
  ktrace_end(a.trace);
}

// ---------------------------------------------------------------- vocab head
struct BVocabArgs {
  CUtensorMap wmap;      // f16 [151936, 1024], box {64, 128}, SWIZZLE_128B
  CUtensorMap xmap;      // f16 [npad, 1024], box {64, npad}, SWIZZLE_128B
  int B;
  int ntiles;            // vocabulary rows / 128
  uint16_t* logits;      // optional [B][ld_logits]
  int64_t ld_logits;
  ArgmaxPartial* part;   // [gridDim.x][64]
  unsigned int* counter;
  int64_t* tokens;       // [B][tok_stride]; tokens[b][pos+1] = argmax
  int64_t tok_stride;
  BatchSeq* seq;         // advanced by the last CTA (pos += 1, n_gen += 1)
  int64_t* token_out;    // optional [B]
  int64_t* amax;         // optional [B][tok_stride]: argmax after every position, prompt included
  int* err;              // optional device error word
  int tag;               // launch tag recorded with a timeout
  unsigned long long* trace;  // optional launch timing record
};

constexpr int kBvAStages = 4;

__host__ __device__ constexpr size_t bvocab_smem_bytes(int npad) {
  return 1024 + (size_t)16 * npad * 128 /* all of x */ + (size_t)kBvAStages * kBgAtomA + 256;
}

template <int NPAD>
__global__ void __launch_bounds__(kBvThreads, 1) k_bvocab(const __grid_constant__ BVocabArgs a) {
  constexpr uint32_t TCOLS = 2 * NPAD <= 32 ? 32 : 2 * NPAD <= 64 ? 64 : 128;  // double buffer
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t x_full, a_full[kBvAStages], a_empty[kBvAStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ float wbv[4][NPAD];
  __shared__ int64_t wbi[4][NPAD];
  __shared__ int is_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t sX = base;                         // 16 atoms of [NPAD x 64]
  ktrace_start(a.trace);
  const uint32_t sA = sX + 16 * NPAD * 128;         // [4][16 KB]
  uint8_t* gbase = smem_raw + (base - smem_u32(smem_raw));

  if (threadIdx.x == 0) {
    mbar_init(&x_full, 1);
    for (int i = 0; i < kBvAStages; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tmem = tmem_base;
  const uint32_t idesc = idesc_f16_f32(128, NPAD);
  const int ntile_mine = (a.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&a.wmap);
      prefetch_tmap(&a.xmap);
      // weights first: they do not depend on the previous kernel
      const int total = ntile_mine * 16;
      int i_done = 0;
      bool x_issued = false;
      for (int i = 0; i < total; ++i) {
        const int t = (int)blockIdx.x + (i >> 4) * (int)gridDim.x, j = i & 15;
        const int s = i % kBvAStages;
        if (i >= kBvAStages &&
            !Q3_BWAIT(&a_empty[s], ((i / kBvAStages) - 1) & 1, kErrTimeoutEmpty, 11))
          break;
        mbar_expect_tx(&a_full[s], kBgAtomA);
        tma_load_2d(gbase + (sA - base) + s * kBgAtomA, &a.wmap, j * 64, t * 128, &a_full[s]);
        i_done = i + 1;
        if (!x_issued && i == kBvAStages - 1) {
          pdl_wait();
          ktrace_release(a.trace);
          mbar_expect_tx(&x_full, 16 * NPAD * 128);
          for (int q = 0; q < 16; ++q) tma_load_2d(gbase + q * NPAD * 128, &a.xmap, q * 64, 0, &x_full);
          x_issued = true;
        }
      }
      if (!x_issued) {
        pdl_wait();
        ktrace_release(a.trace);
        mbar_expect_tx(&x_full, 16 * NPAD * 128);
        for (int q = 0; q < 16; ++q) tma_load_2d(gbase + q * NPAD * 128, &a.xmap, q * 64, 0, &x_full);
      }
      // the CTA may not exit before every issued copy has landed
      Q3_BWAIT(&x_full, 0, kErrTimeoutFull, 12);
      for (int st = 0; st < kBvAStages && st < i_done; ++st)
        Q3_BWAIT(&a_full[st], ((i_done - 1 - st) / kBvAStages) & 1, kErrTimeoutFull, 13);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = Q3_BWAIT(&x_full, 0, kErrTimeoutFull, 14);
      int i = 0;
      for (int k = 0; ok && k < ntile_mine; ++k) {
        const int ab = k & 1;
        if (k >= 2 && !Q3_BWAIT(&acc_empty[ab], ((k / 2) - 1) & 1, kErrTimeoutEmpty, 15)) break;
        tc_fence_after();
        for (int j = 0; j < 16; ++j, ++i) {
          const int s = i % kBvAStages;
          if (!Q3_BWAIT(&a_full[s], (i / kBvAStages) & 1, kErrTimeoutFull, 16)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t aa = sA + s * kBgAtomA, xx = sX + j * NPAD * 128;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tmem + ab * NPAD, sw128_desc(aa + 32 * kk), sw128_desc(xx + 32 * kk), idesc,
                     (j | kk) != 0);
          umma_commit(&a_empty[s]);
        }
        umma_commit(&acc_full[ab]);
      }
      umma_commit(&mma_done);
      Q3_BWAIT(&mma_done, 0, kErrTimeoutFull, 17);  // no MMA in flight at dealloc
    }
  } else {
    // epilogue warps: per sequence, the best (value, index) of this CTA;
    // lane j of a warp keeps the candidates of sequences j, j+32.
    const int q = warp & 3;
    const uint32_t lane_base = (32u * q) << 16;
    constexpr int PER_LANE = (NPAD + 31) / 32;
    float bv[PER_LANE];
    int64_t bi[PER_LANE];
#pragma unroll
    for (int k = 0; k < PER_LANE; ++k) {
      bv[k] = -__int_as_float(0x7f800000);
      bi[k] = -1;
    }
    pdl_wait();
    for (int k = 0; k < ntile_mine; ++k) {
      const int t = (int)blockIdx.x + k * (int)gridDim.x;
      const int ab = k & 1;
      if (!Q3_BWAIT(&acc_full[ab], (k / 2) & 1, kErrTimeoutFull, 18)) break;
      tc_fence_after();
      const int64_t n = (int64_t)t * 128 + 32 * q + lane;  // this lane's vocabulary row
#pragma unroll
      for (int col0 = 0; col0 < NPAD; col0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + lane_base + ab * NPAD + col0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int b = col0 + j;
          const uint16_t lh = f2h(__uint_as_float(v[j]));
          if (a.logits != nullptr && b < a.B) a.logits[(int64_t)b * a.ld_logits + n] = lh;
          // warp argmax over its 32 rows in one reduction: the key orders as
          // the f16 value (-0 taken as +0: they compare equal) and then by
          // lower row; NaN and -inf never win (key 0), as in the strict ogt
          // scan (model/qwen3_full.mlir:1482-1507)
          const uint32_t hz = lh == 0x8000u ? 0u : (uint32_t)lh;
          const bool nan_or_ninf = (hz & 0x7C00u) == 0x7C00u && ((hz & 0x03FFu) != 0u || (hz & 0x8000u));
          const uint32_t ord = (hz & 0x8000u) ? (~hz & 0xFFFFu) : (hz | 0x8000u);
          const uint32_t key = nan_or_ninf ? 0u : ((ord << 16) | (0xFFFFu - (uint32_t)lane));
          const uint32_t best = __reduce_max_sync(0xffffffffu, key);
          if (lane == (b & 31) && best != 0u) {
            const uint32_t bo = best >> 16;
            const uint16_t bh = (bo & 0x8000u) ? (uint16_t)(bo & 0x7FFFu) : (uint16_t)(~bo & 0xFFFFu);
            const int64_t li = (int64_t)t * 128 + 32 * q + (int64_t)(0xFFFFu - (best & 0xFFFFu));
            const float lv = h2f(bh);
            if (am_better(lv, li, bv[b >> 5], bi[b >> 5])) {
              bv[b >> 5] = lv;
              bi[b >> 5] = li;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
#pragma unroll
    for (int k = 0; k < PER_LANE; ++k) {
      const int b = lane + 32 * k;
      if (b < NPAD) {
        wbv[q][b] = bv[k];
        wbi[q][b] = bi[k];
      }
    }
  }
  __syncwarp();  // reconverge the role-diverged warps before the CTA barrier
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TCOLS);
  }
  // CTA candidate per sequence, then the last CTA reduces all of them
  if (threadIdx.x < NPAD) {
    const int b = threadIdx.x;
    float v = -__int_as_float(0x7f800000);
    int64_t ii = -1;
    for (int w = 0; w < 4; ++w)
      if (am_better(wbv[w][b], wbi[w][b], v, ii)) {
        v = wbv[w][b];
        ii = wbi[w][b];
      }
    a.part[(int64_t)blockIdx.x * kBMaxBatch + b].v = v;
    a.part[(int64_t)blockIdx.x * kBMaxBatch + b].i = ii;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.counter, 1u);
    is_last = (prev == gridDim.x - 1);
    if (is_last) *a.counter = 0u;
  }
  __syncthreads();
  ktrace_end(a.trace);
  if (!is_last) return;
  __threadfence();
  // The candidates of every CTA, [c][b] for b < B, brought into the (now
  // idle) dynamic shared memory by all threads' 16-byte cp.async at once;
  // thread (b, g) then scans CTAs c = g mod 3 and thread b folds the three
  // (any order: am_better is a total order).
  const int nc = (int)gridDim.x;
  uint8_t* const stage = smem_raw + (((smem_u32(smem_raw) + 1023u) & ~1023u) - smem_u32(smem_raw));
  const bool staged = (size_t)nc * NPAD * sizeof(ArgmaxPartial) <= bvocab_smem_bytes(NPAD) - 1024 - 256 &&
                      (reinterpret_cast<uintptr_t>(a.part) & 15) == 0;
  if (staged) {
    for (int f = threadIdx.x; f < nc * NPAD; f += kBvThreads) {
      const int c = f / NPAD, b = f - c * NPAD;
      if (b < a.B)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(stage + (size_t)f * 16)),
                     "l"(a.part + (int64_t)c * kBMaxBatch + b)
                     : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
  __syncthreads();
  constexpr int kGroups = kBvThreads / 64;
  {
    const int b = threadIdx.x & 63, g = threadIdx.x >> 6;
    float v = -__int_as_float(0x7f800000);
    int64_t ii = -1;
    if (b < a.B) {
      for (int c = g; c < nc; c += kGroups) {
        float pv;
        int64_t pi;
        if (staged) {
          const ArgmaxPartial* p = reinterpret_cast<const ArgmaxPartial*>(stage + (size_t)(c * NPAD + b) * 16);
          pv = p->v;
          pi = p->i;
        } else {
          const ArgmaxPartial* p = a.part + (int64_t)c * kBMaxBatch + b;
          pv = __ldcg(&p->v);
          pi = __ldcg(reinterpret_cast<const long long*>(&p->i));
        }
        if (am_better(pv, pi, v, ii)) {
          v = pv;
          ii = pi;
        }
      }
      wbv[g][b] = v;
      wbi[g][b] = ii;
    }
  }
  __syncthreads();
  if (threadIdx.x < a.B) {
    const int b = threadIdx.x;
    float v = wbv[0][b];
    int64_t ii = wbi[0][b];
#pragma unroll
    for (int g = 1; g < kGroups; ++g)
      if (am_better(wbv[g][b], wbi[g][b], v, ii)) {
        v = wbv[g][b];
        ii = wbi[g][b];
      }
    if (a.token_out != nullptr) a.token_out[b] = ii;
    if (a.seq != nullptr) {
      BatchSeq& s = a.seq[b];
      if (s.pos < 0 || s.pos + 1 >= a.tok_stride) {  // no room for the next token
        if (a.err) atomicCAS(a.err, 0, kErrBadPos);
      } else {
        if (a.amax != nullptr) a.amax[(int64_t)b * a.tok_stride + s.pos + 1] = ii;
        if (s.pos + 1 >= s.n_prompt) {  // past the prompt: the argmax is the next token
          a.tokens[(int64_t)b * a.tok_stride + s.pos + 1] = ii;
          s.n_gen += 1;
        }
        s.pos += 1;
      }
    }
  }
}

}  // namespace q3
