// q3_fused.cuh -- one decoder layer (model/qwen3_full.mlir:751-864) of the
// batch-1 decode step as TWO cluster kernels, for the fused engine.
//
// Every dependency between the five projections of a layer costs a grid-wide
// hand-off (~1 us on B200 for a kernel boundary under programmatic dependent
// launch, ~1.3 us for a grid barrier), so the layer is cut at the only two
// points where every output needs every input:
//
//   k_fused_attn   one 16-CTA cluster per kv head h (q heads 2h, 2h+1):
//                  x = f16(h1 + f16(sum_c dpart[c]))  (previous layer's down)
//                  -> RMSNorm -> this head pair's 512 Q|K|V rows (32 per CTA)
//                  -> rows gathered over DSMEM -> QK-norm + RoPE -> K/V row
//                  written at slot layer*S + pos -> attention over the cache,
//                  chunks of 32 keys spread over the cluster, folded over DSMEM
//                  -> the head pair's slice of W_o (K columns 256h..256h+255,
//                  64 rows per CTA) as an f32 partial opart[h][1024].
//   k_fused_ffn    one 16-CTA cluster per 384-wide slice c of the FFN:
//                  h1 = f16(x + f16(sum_h opart[h])) -> RMSNorm -> 24 gate and
//                  24 up rows per CTA -> SwiGLU -> the slice's 384 act values
//                  gathered over DSMEM -> W_down columns 384c..384c+383 (64 rows
//                  per CTA) as an f32 partial dpart[c][1024].
//
// The O and down projections are therefore split along K (by head pair and by
// FFN slice); their 8 partials are summed in index order by the consumer, in
// f32, before the f16 rounding and the residual add of the reference.  All
// other arithmetic (RMSNorm, Q|K|V and gate|up row dots, QK-norm, RoPE,
// SwiGLU) is the per-row order of the exact engine.  Each order is stated
// below and restated by the CPU oracle (q3o_layer with Q3O_ORDER_FUSED), so
// the engine is compared with it bit for bit.
//
// Weights never depend on the previous kernel: every CTA issues its bulk
// copies (Q8_0 rows in the reference layout, 16-byte aligned windows) and the
// copies of its cached K/V chunks before griddepcontrol.wait.  Shared memory
// and registers are sized so that one CTA of each kernel fits on an SM
// together, which lets the next kernel's copies stream under this one.
#pragma once

#include "q3_attn.cuh"
#include "q3_common.cuh"
#include "q3_gemv.cuh"
#include "q3_tc.cuh"

namespace q3 {

constexpr int kFC = 16;     // CTAs per cluster

// ---- k_fused_attn
constexpr int kFaThreads = 256;
constexpr int kFaQRows = 2 * kHD / kFC;              // 16 q rows of the head pair per CTA
constexpr int kFaKRows = kHD / kFC;                  // 8 k rows and 8 v rows per CTA
constexpr int kFaRows = kFaQRows + 2 * kFaKRows;     // 32
constexpr uint32_t kRow1K = (kDim / kQBlk) * kQBytes;  // 1088: a K = 1024 Q8_0 row
constexpr int kFaORows = kDim / kFC;                 // 64 rows of W_o per CTA
constexpr uint32_t kORowBytes = (2 * kDim / kQBlk) * kQBytes;  // 2176: a W_o row
constexpr uint32_t kFaOBytes = 8 * kQBytes;          // 272: a W_o row's 8 blocks of one head pair
constexpr int kFaAttWarps = 8;                       // every warp owns a K/V chunk slot
constexpr int kFaChunk = 8;                          // keys per attention chunk
// A chunk's K tile: two SWIZZLE_128B boxes of 8 keys x 64 dims (one 1024-byte
// swizzle atom each; the 16-byte reads of 8 keys are bank-conflict free); its
// V tile: one plain box of 8 keys x 128 dims.  Slots are 1024-byte aligned.
constexpr uint32_t kFaKHalf = kFaChunk * 64 * 2;       // 1024
constexpr uint32_t kFaKTile = 2 * kFaKHalf;            // 2048
constexpr uint32_t kFaVTile = kFaChunk * kHD * 2;      // 2048
constexpr uint32_t kFaSlot = kFaKTile + kFaVTile;      // 4096
constexpr uint32_t kFaWqkvBytes = kFaRows * kRow1K;          // 34816
constexpr uint32_t kFaWoBytes = kFaORows * kFaOBytes;        // 17408
// dynamic shared memory: K/V slots first (aligned), then the weights
constexpr uint32_t kFaSmem = 1024 + kFaAttWarps * kFaSlot + kFaWqkvBytes + kFaWoBytes;  // 85248
constexpr int kFaMaxPasses = 4;  // chunks per warp: caches up to 4 * 8 * 16 * 8 = 4096 positions
constexpr int64_t kFusedMaxPositions = (int64_t)kFaMaxPasses * kFaAttWarps * kFC * kFaChunk;

// ---- k_fused_ffn
constexpr int kFbThreads = 384;                      // 12 warps
constexpr int kFbSlice = kFFN / kFParts;             // 384 act values per cluster
constexpr int kFbAct = kFbSlice / kFC;               // 24 per CTA
constexpr int kFbDRows = kDim / kFC;                 // 64 rows of W_down per CTA
constexpr int kFbDBlocks = kFbSlice / kQBlk;         // 12 blocks of each row
constexpr uint32_t kDRowBytes = (kFFN / kQBlk) * kQBytes;  // 3264: a W_down row
constexpr uint32_t kFbDWin = 416;                    // 16-byte window holding 12 blocks (408 B)
constexpr uint32_t kFbGUBytes = kFbAct * kRow1K;     // 26112 (gate rows; the same for up rows)
constexpr uint32_t kFbDBytes = kFbDRows * kFbDWin;   // 26624
constexpr uint32_t kFbSmem = 2 * kFbGUBytes + kFbDBytes;  // 78848

static_assert(kFaThreads == 2 * kHD, "the attention fold maps one thread to one output value");
static_assert(kFbAct * kFC * kFParts == kFFN, "FFN slices");
static_assert(kFbThreads / 32 * 2 == kFbAct, "two act values per warp");

struct FaArgs {
  // W_o of all layers as u32 [28*1024 rows, 544] (box {68, 64}: a head
  // pair's 272-byte slice of 64 rows); the K cache as f16 [slots, 1024] (box
  // {64, 32}, SWIZZLE_128B) and the V cache (box {128, 32})
  CUtensorMap wo_map;
  CUtensorMap k_map;
  CUtensorMap v_map;
  int layer;
  const uint8_t* wq;          // this layer's W_q [2048, 1024] Q8_0 (reference layout)
  const uint8_t* wk;          // W_k [1024, 1024]
  const uint8_t* wv;          // W_v [1024, 1024]
  const uint16_t* attn_norm;  // [1024]
  const uint16_t* q_norm;     // [128]
  const uint16_t* k_norm;     // [128]
  // residual stream in: with tokens (layer 0) x = embd[tokens[pos]]; else
  // x = f16(h1 + f16(dpart[0] + ... + dpart[7])), or x = h1 without dpart
  const uint16_t* h1;
  const float* dpart;         // [8][1024]
  const int64_t* tokens;
  const uint16_t* embd;
  uint16_t* x_out;            // x, written by CTA 0 (the ffn kernel's residual)
  float* opart;               // out: [8][1024] O partials (one per head pair)
  uint16_t* kc;               // flat K cache [slots, 8, 128]
  uint16_t* vc;
  const float* rope_cos;      // [S, 64]
  const float* rope_sin;
  int64_t slot0;              // layer * S
  int64_t S;
  const int64_t* pos;         // device position (read before the dependency wait)
  const int32_t* stop;        // optional: the step is skipped when *stop != 0
  int* err;
  unsigned long long* trace;  // optional launch timing record
  long long* phase;           // optional per-CTA phase stamps [grid][kFPhases] (ns)
};

struct FbArgs {
  CUtensorMap wd_map;         // W_down of all layers as u32 [28*1024 rows, 816], box {104, 64}
  int layer;
  const uint8_t* wgu;         // this layer's W_gate|up [6144, 1024] (gate rows, then up rows)
  const uint16_t* ffn_norm;   // [1024]
  const uint16_t* x;          // residual (the attention kernel's x_out)
  const float* opart;         // [8][1024]
  uint16_t* h1_out;           // h1, written by CTA 0 (the next layer's residual)
  float* dpart;               // out: [8][1024] down partials (one per FFN slice)
  const int32_t* stop;        // optional: the step is skipped when *stop != 0
  SeqState* advance;          // if set, pos += 1 (the last kernel of a prompt-ingestion step)
  int* err;
  unsigned long long* trace;
  long long* phase;           // optional per-CTA phase stamps [grid][kFPhases] (ns)
};

// Phase stamps (latency analysis): thread 0 of each CTA records %globaltimer
// at the end of each numbered step of the kernels below.
constexpr int kFPhases = 16;
__device__ __forceinline__ void fphase(long long* p, int k) {
  if (p != nullptr && threadIdx.x == 0) {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    p[blockIdx.x * kFPhases + k] = t;
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 16-byte asynchronous copy global -> shared (L2 only, like __ldcg); the
// thread's copies are complete after cp_async_wait_all.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Four warp sums (warp_sum's butterfly on each value), the shuffles of the
// four interleaved: the same operations per value, four chains in flight.
__device__ __forceinline__ void warp_sum4(float (&v)[4]) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(v[j], __shfl_xor_sync(0xffffffffu, v[j], off));
}

// Four row dots of one lane's block (block b = lane, K = 1024) in the block
// order of q8_block_dot_mlir, the four inner chains interleaved:
// out[j] = fma(scale_j, inner_j, 0) with inner_j = the 32 products in order.
__device__ __forceinline__ void q8_block_dot4_mlir(const Q8BlockWords (&b)[4], const uint32_t (&xr)[16],
                                                   float (&out)[4]) {
  float inner[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t h01, h23;
      q8x4_to_h2(b[j].q[i], h01, h23);
      inner[j] = fma_h2(h01, xr[2 * i], inner[j]);
      inner[j] = fma_h2(h23, xr[2 * i + 1], inner[j]);
    }
#pragma unroll
  for (int j = 0; j < 4; ++j) out[j] = __fmaf_rn(h2f((uint16_t)b[j].scale16), inner[j], 0.0f);
}

// A K = 1024 x block (32 f16) from shared memory in the 40-half block layout.
__device__ __forceinline__ void load_xblock(const uint16_t* xs, int b, uint32_t (&xb)[16]) {
  const uint4* p = reinterpret_cast<const uint4*>(xs + b * kXhStride);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint4 t = p[v];
    xb[4 * v] = t.x, xb[4 * v + 1] = t.y, xb[4 * v + 2] = t.z, xb[4 * v + 3] = t.w;
  }
}

// Per-head RMSNorm + NeoX RoPE (head_norm_rope's operations) of a head held in
// shared memory.
__device__ __forceinline__ void head_norm_rope_smem(const uint16_t* x, const uint16_t (&gv)[4],
                                                    float c0, float s0, float c1, float s1,
                                                    int lane, uint16_t* dst) {
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = h2f(x[lane + 32 * i]);
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = __fmaf_rn(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float r = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), kEps));
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = h2f(f2h(__fmul_rn(__fdiv_rn(v[i], r), h2f(gv[i]))));
  dst[lane] = f2h(__fsub_rn(__fmul_rn(n[0], c0), __fmul_rn(n[2], s0)));
  dst[lane + 64] = f2h(__fadd_rn(__fmul_rn(n[0], s0), __fmul_rn(n[2], c0)));
  dst[lane + 32] = f2h(__fsub_rn(__fmul_rn(n[1], c1), __fmul_rn(n[3], s1)));
  dst[lane + 96] = f2h(__fadd_rn(__fmul_rn(n[1], s1), __fmul_rn(n[3], c1)));
}

// ---------------------------------------------------------------------------
// Cluster exchanges.  Every exchange is a push: the producer stores 16-byte
// pieces into the consumers' shared memory with st.async, whose arrival
// counts bytes on the consumer's own mbarrier; a consumer waits for its
// expected byte count and nothing else (no cluster barrier after the release).
// ---------------------------------------------------------------------------
constexpr int kFSlice = kDim / kFC;  // 64 residual-stream elements rebuilt per rank
constexpr uint32_t kFSliceBytes = kFC * (kFSlice * 2 + 16);  // 64 values + (ss, 0, 0, 0) from each rank

// Rank r's slice of the residual stream and its sum of squares, by warp 0
// (lanes 0-15 hold 4 elements each, v): stored into yloc, pushed with the
// slice's sum of squares to every rank (xr[64 r ..], xss[r]).  The slice's
// sum of squares: each lane's fma chain over its 4 elements, then
// v += shfl_xor(v, 8), (4), (2), (1) over the 16 lanes.  Warp 0 only.
__device__ __forceinline__ void push_slice(uint2 v, int r, int lane, uint16_t* yloc, uint16_t* xr,
                                           float4* xss, uint4* ssl, uint64_t* bar) {
  float acc = 0.0f;
  const float e[4] = {h2f((uint16_t)(v.x & 0xffffu)), h2f((uint16_t)(v.x >> 16)),
                      h2f((uint16_t)(v.y & 0xffffu)), h2f((uint16_t)(v.y >> 16))};
#pragma unroll
  for (int i = 0; i < 4; ++i) acc = __fmaf_rn(e[i], e[i], acc);
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  if (lane < 16) *reinterpret_cast<uint2*>(yloc + 4 * lane) = v;
  if (lane == 0) *ssl = make_uint4(__float_as_uint(acc), 0u, 0u, 0u);
  __syncwarp();
  for (int i = lane; i < 9 * kFC; i += 32) {
    const int dst = i / 9, piece = i % 9;
    const uint4 val = piece < 8 ? reinterpret_cast<const uint4*>(yloc)[piece] : *ssl;
    const uint32_t at = piece < 8 ? smem_u32(xr + kFSlice * r + 8 * piece) : smem_u32(&xss[r]);
    st_async_v4(at, (uint32_t)dst, val, smem_u32(bar));
  }
}

// RMSNorm of the gathered x (xr) with gamma gam (shared memory) into xs
// (block layout): ss = ((ss_0 + ss_1) + ...) + ss_15 over the ranks' slice
// sums, r = sqrt(ss/1024 + eps), y = f16((x / r) * g).  Threads 0-255.
__device__ __forceinline__ void slice_rmsnorm(const uint16_t* xr, const float4* xss,
                                              const uint16_t* gam, uint16_t* xs) {
  if (threadIdx.x < 256) {
    float ss = xss[0].x;
#pragma unroll
    for (int q = 1; q < kFC; ++q) ss = __fadd_rn(ss, xss[q].x);
    const float rn = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kDim), kEps));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = threadIdx.x + 256 * i;
      xs[xh_index(k)] = rms_apply(xr[k], gam[k], rn);
    }
  }
  __syncthreads();
}

// ===========================================================================
// k_fused_attn: grid 8 clusters x 16 CTAs, 256 threads.
// ===========================================================================
// Attention order (restated by q3o_attention_fused): chunk ci (keys 32ci ..
// 32ci+31 of 0..pos) belongs to cluster rank ci % 16 as its local chunk
// j = ci / 16.  A chunk gives, per q head, m = max s_t, p_t = exp(s_t - m),
// l = butterfly sum of p_t, o_d = fma chain of p_t * v_td over t in order
// (s_t = (fma chain of q_d * k_td over d) * rsqrt(128)).  Rank r folds its
// chunks: M_r = max_j m_j, e_j = exp(m_j - M_r), l_r = fma chain of l_j * e_j
// over j, o_r = fma chain of o_j * e_j.  The cluster folds the ranks the same
// way (M = max M_r, E_r = exp(M_r - M), chains over r = 0..15) and
// out_d = f16(O_d / L); rank q folds output dims 16q .. 16q+15.  A rank
// without chunks contributes M_r = -inf.
__global__ void __launch_bounds__(kFaThreads, 1) k_fused_attn(const __grid_constant__ FaArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* kvs = smem_raw + (((smem_u32(smem_raw) + 1023u) & ~1023u) - smem_u32(smem_raw));
  uint8_t* wqkv = kvs + kFaAttWarps * kFaSlot;
  uint8_t* wo = wqkv + kFaWqkvBytes;
  __shared__ __align__(16) uint16_t xr[kDim];
  __shared__ __align__(16) float4 xss[kFC];
  __shared__ __align__(16) uint16_t yloc[kFSlice];
  __shared__ __align__(16) uint4 ssl;
  __shared__ __align__(16) uint16_t xs[kDim / kQBlk * kXhStride];
  __shared__ __align__(16) uint16_t loc[kFaRows];
  __shared__ __align__(16) uint16_t rstage_h[kFSlice];          // warp 0's residual slice
  __shared__ __align__(16) float rstage_p[kFParts][kFSlice];    // and its 8 partials
  __shared__ __align__(16) uint16_t qkv_h[4 * kHD];  // q head 2h | q head 2h+1 | k | v (raw)
  __shared__ __align__(16) uint16_t qs[2][kHD];
  __shared__ __align__(16) uint16_t ks[kHD];
  __shared__ __align__(16) AttnPartial part[kFaAttWarps][2];  // each warp's running fold
  __shared__ __align__(16) AttnPartial cpart[2];
  // this rank's share of the cluster fold: from every rank q, (M, l, -, -,
  // o[16 dims]) of the output dims 16r .. 16r+15 of the head pair
  __shared__ __align__(16) float fin[kFC][20];
  __shared__ __align__(16) uint16_t fout[16];
  __shared__ __align__(16) uint16_t att[2 * kHD / kQBlk * kXhStride];
  __shared__ __align__(8) uint64_t wbar, obar, cbar, kvbar[kFaAttWarps], xbar, qbar, fbar, abar;
  __shared__ __align__(16) float rope_c[64], rope_s[64];      // RoPE angles at pos
  __shared__ __align__(16) uint16_t qkn[2][kHD];              // q_norm, k_norm gammas
  __shared__ __align__(16) uint16_t gam[kDim];                // attn_norm gamma

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x / kFC;
  const int r = (int)cluster_rank();
  ktrace_start(a.trace);
  fphase(a.phase, 0);
  if (tid == 0) {
    mbar_init(&wbar, 1);
    mbar_init(&obar, 1);
    mbar_init(&cbar, 1);
    for (int i = 0; i < kFaAttWarps; ++i) mbar_init(&kvbar[i], 1);
    mbar_init(&xbar, 1);
    mbar_init(&qbar, 1);
    mbar_init(&fbar, 1);
    mbar_init(&abar, 1);
    fence_mbar_init();
    // the bytes each exchange brings in from the 16 ranks
    mbar_expect_tx(&xbar, kFSliceBytes);
    mbar_expect_tx(&qbar, kFC * 4 * 16);
    mbar_expect_tx(&fbar, kFC * 5 * 16);
    mbar_expect_tx(&abar, kFC * 2 * 16);
  }
  __syncthreads();
  pdl_launch_dependents();
  // The decode state changes only in a step's last kernel, and every step is
  // its own graph launch: read it before the wait.  It is the same for every
  // CTA, so a CTA that returns here takes its whole cluster with it.
  const int stop = a.stop != nullptr ? *a.stop : 0;
  const int64_t pos = *a.pos;
  if (stop != 0) return;
  if (pos < 0 || pos >= a.S || pos >= kFusedMaxPositions) {
    if (tid == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    return;
  }
  const int64_t T = pos + 1;
  const int nch = (int)((T + kFaChunk - 1) / kFaChunk);
  const int nloc = r < nch ? (nch - 1 - r) / kFC + 1 : 0;  // local chunks j: ci = r + 16 j
  cluster_sync_all();  // every rank's exchange barriers are initialised

  // ---- copies that do not depend on the previous kernel
  const uint64_t pol_w = l2_policy_evict_first();
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&a.wo_map);
    prefetch_tmap(&a.k_map);
    prefetch_tmap(&a.v_map);
    mbar_expect_tx(&wbar, kFaWqkvBytes);
    bulk_g2s(wqkv, a.wq + (int64_t)(2 * kHD * h + kFaQRows * r) * kRow1K, kFaQRows * kRow1K,
             &wbar, pol_w);
    bulk_g2s(wqkv + kFaQRows * kRow1K, a.wk + (int64_t)(kHD * h + kFaKRows * r) * kRow1K,
             kFaKRows * kRow1K, &wbar, pol_w);
    bulk_g2s(wqkv + (kFaQRows + kFaKRows) * kRow1K,
             a.wv + (int64_t)(kHD * h + kFaKRows * r) * kRow1K, kFaKRows * kRow1K, &wbar, pol_w);
  }
  // local chunk j (keys 8 (r + 16 j) ..) into warp w's slot: whole boxes;
  // rows past pos are never used, rows past the cache read as zeros
  auto issue_chunk = [&](int w, int j) {
    if (lane == 0) {
      const int y = (int)(a.slot0 + (int64_t)(r + kFC * j) * kFaChunk);
      uint8_t* slot = kvs + w * kFaSlot;
      mbar_expect_tx(&kvbar[w], kFaSlot);
      tma_load_2d(slot, &a.k_map, kHD * h, y, &kvbar[w]);
      tma_load_2d(slot + kFaKHalf, &a.k_map, kHD * h + 64, y, &kvbar[w]);
      tma_load_2d(slot + kFaKTile, &a.v_map, kHD * h, y, &kvbar[w]);
    }
    __syncwarp();
  };
  if (warp < kFaAttWarps && warp < nloc) issue_chunk(warp, warp);

  // constants: gammas, RoPE angles at pos, the layer-0 embedding slice
  // Constants (gammas, RoPE angles at pos, the layer-0 embedding slice) come
  // by bulk copy into shared memory: no register waits on them before the
  // release (values loaded into registers there were measured to arrive only
  // after it).
  if (warp == 2 && lane == 0) {
    const uint64_t pol_c = l2_policy_evict_normal();
    int64_t tok = 0;
    if (a.tokens != nullptr) {
      tok = a.tokens[pos];
      if (tok < 0 || tok >= kVocab) {
        if (a.err) atomicCAS(a.err, 0, kErrBadToken);
        tok = 0;
      }
    }
    mbar_expect_tx(&cbar, kDim * 2 + 2 * kHD * 2 + 2 * 64 * 4 + (a.tokens != nullptr ? kFSlice * 2 : 0));
    bulk_g2s(gam, a.attn_norm, kDim * 2, &cbar, pol_c);
    bulk_g2s(qkn[0], a.q_norm, kHD * 2, &cbar, pol_c);
    bulk_g2s(qkn[1], a.k_norm, kHD * 2, &cbar, pol_c);
    bulk_g2s(rope_c, a.rope_cos + pos * 64, 64 * 4, &cbar, pol_c);
    bulk_g2s(rope_s, a.rope_sin + pos * 64, 64 * 4, &cbar, pol_c);
    if (a.tokens != nullptr)
      bulk_g2s(yloc, a.embd + tok * (int64_t)kDim + kFSlice * r, kFSlice * 2, &cbar, pol_c);
  }
  const int k0 = kFSlice * r + 4 * (lane & 15);  // warp 0: this lane's 4 slice elements

  fphase(a.phase, 11);
  pdl_wait();  // the previous kernel's outputs (h1, dpart) are visible
  ktrace_release(a.trace);
  fphase(a.phase, 1);

  bool ok = mbar_wait_own(&cbar, 0u, a.err, kErrTimeoutFull);  // constants (long landed)
  // 1) this rank's slice of x (cluster 0 publishes it): warp 0 starts the
  //    slice's loads as asynchronous copies and sums them after its rows'
  //    conversion below
  const bool staged = a.tokens == nullptr;
  if (warp == 0 && staged) {
    if (lane < 8) cp_async16(rstage_h + 8 * lane, a.h1 + kFSlice * r + 8 * lane);
    if (a.dpart != nullptr && lane < 16) {
#pragma unroll
      for (int c = 0; c < kFParts; ++c) cp_async16(&rstage_p[c][4 * lane], a.dpart + c * kDim + k0);
    }
  }
  // 2) this warp's rows w, w+8 (q), w+16 (k), w+24 (v) at block `lane`
  //    converted to exact half2 registers (warp 0's while its copies travel)
  const bool wok = mbar_wait_own(&wbar, 0u, a.err, kErrTimeoutFull);
  uint32_t hq[4][1][16];
  float sq[4][1];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    q8_row_to_h2regs<1>(smem_u32(wqkv) + (warp + 8 * i) * kRow1K, kDim / kQBlk, lane, hq[i], sq[i]);
  // 3) warp 0: the slice x = f16(h1 + f16(sum_c dpart[c])), pushed with its
  //    sum of squares (resid_plus_parts' operations)
  if (warp == 0) {
    if (staged) {
      cp_async_wait_all();
      __syncwarp();
    }
    uint2 xv = make_uint2(0u, 0u);
    if (lane < 16) {
      if (!staged) {
        xv = *reinterpret_cast<const uint2*>(yloc + 4 * lane);
      } else {
        const uint2 rv = *reinterpret_cast<const uint2*>(rstage_h + 4 * lane);
        if (a.dpart == nullptr) {
          xv = rv;
        } else {
          xv = resid_finish_smem(rv, smem_u32(&rstage_p[0][4 * lane]), kFSlice * 4);
        }
      }
    }
    __syncwarp();
    if (h == 0 && lane < 16) *reinterpret_cast<uint2*>(a.x_out + k0) = xv;
    push_slice(xv, r, lane, yloc, xr, xss, &ssl, &xbar);
  }
  fphase(a.phase, 3);
  ok = mbar_wait_own(&xbar, 0u, a.err, kErrTimeoutFull) && ok;
  // 4) RMSNorm with attn_norm
  slice_rmsnorm(xr, xss, gam, xs);
  fphase(a.phase, 2);
  // the W_o slice is needed last: its copy goes out now, so that no weight
  // bytes are in flight while the residual slices are read from L2
  if (warp == 1 && lane == 0) {
    mbar_expect_tx(&obar, kFaWoBytes);
    tma_load_2d(wo, &a.wo_map, (int)(kFaOBytes / 4) * h, a.layer * kDim + kFaORows * r, &obar);
  }
  // 5) Q|K|V dots (the block order of q8_block_dot_mlir; q8_h2regs_dot_xh's
  //    operations for each row, the four rows' chains interleaved)
  {
    const uint4* xb = reinterpret_cast<const uint4*>(xs + lane * kXhStride);
    float inner[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 xv = xb[q];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        inner[i] = fma_h2(hq[i][0][4 * q + 0], xv.x, inner[i]);
        inner[i] = fma_h2(hq[i][0][4 * q + 1], xv.y, inner[i]);
        inner[i] = fma_h2(hq[i][0][4 * q + 2], xv.z, inner[i]);
        inner[i] = fma_h2(hq[i][0][4 * q + 3], xv.w, inner[i]);
      }
    }
    float d[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = __fmaf_rn(sq[i][0], inner[i], 0.0f);
    warp_sum4(d);
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) loc[warp + 8 * i] = f2h(d[i]);
    }
  }
  __syncthreads();
  fphase(a.phase, 4);
  // 6) every rank pushes its rows into every rank's copy of the head pair's
  //    raw q (2 x 128) | k | v: q rows 16r.., k rows 8r.., v rows 8r..
  if (tid < 4 * kFC) {
    const int dst = tid >> 2, piece = tid & 3;
    const uint4 v = reinterpret_cast<const uint4*>(loc)[piece];
    const int at = piece < 2 ? kFaQRows * r + 8 * piece
                             : (piece == 2 ? 2 * kHD : 3 * kHD) + kFaKRows * r;
    st_async_v4(smem_u32(qkv_h + at), (uint32_t)dst, v, smem_u32(&qbar));
  }
  ok = mbar_wait_own(&qbar, 0u, a.err, kErrTimeoutFull) && ok;
  fphase(a.phase, 5);
  // 7) QK-norm + RoPE: q heads by warps 0, 1; the k head by warp 2
  if (warp < 3) {
    uint16_t gv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) gv[i] = qkn[warp < 2 ? 0 : 1][lane + 32 * i];
    head_norm_rope_smem(qkv_h + (warp < 2 ? warp : 2) * kHD, gv, rope_c[lane], rope_s[lane],
                        rope_c[lane + 32], rope_s[lane + 32], lane, warp < 2 ? qs[warp] : ks);
  }
  __syncthreads();
  fphase(a.phase, 6);
  // the new K (normed, roped) and V (raw) rows at slot layer*S + pos
  if (r == 0 && tid < kHD) {
    const int64_t off = (a.slot0 + pos) * (kNKV * kHD) + h * kHD + tid;
    a.kc[off] = ks[tid];
    a.vc[off] = qkv_h[3 * kHD + tid];
  }

  // 8) this rank's chunks: warp w takes local chunks w, w+8, ... through its
  //    slot and folds them as it goes (att_merge order); lane = 8 q + key
  //    for the scores (dims 32q .. 32q+31 of the key), lane = 4 head dims for p.v
  bool kvok = true;
  {
    const uint32_t slot = smem_u32(kvs + warp * kFaSlot);
    const int key = lane & 7, qd = lane >> 3;
    float m0 = -__int_as_float(0x7f800000), m1 = m0, l0 = 0.0f, l1 = 0.0f;
    float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
    int pass = 0;
    for (int j = warp; j < nloc; j += kFaAttWarps, ++pass) {
      kvok = mbar_wait_own(&kvbar[warp], (uint32_t)(pass & 1), a.err, kErrTimeoutFull) && kvok;
      if (j == 0) fphase(a.phase, 7);
      const int64_t t0 = (int64_t)(r + kFC * j) * kFaChunk;
      const int64_t t = t0 + key;
      const bool valid = t < T;
      float s0 = -__int_as_float(0x7f800000), s1 = s0;
      {
        // dims 32 qd .. 32 qd + 31 = 16-byte chunks 4 qd .. 4 qd + 3 of the key:
        // the new key from ks, cached keys from the swizzled tile
        const uint4* q0 = reinterpret_cast<const uint4*>(qs[0]);
        const uint4* q1 = reinterpret_cast<const uint4*>(qs[1]);
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int v = 4 * qd + i;
          uint4 kv;
          if (t == pos) {
            kv = reinterpret_cast<const uint4*>(ks)[v];
          } else {
            const uint32_t ad = slot + (v >> 3) * kFaKHalf + sw128_chunk_offset((uint32_t)key, (uint32_t)(v & 7));
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(kv.x), "=r"(kv.y), "=r"(kv.z), "=r"(kv.w) : "r"(ad));
          }
          const uint4 x0 = q0[v], x1 = q1[v];
          a0 = fma_h2(x0.x, kv.x, a0);
          a0 = fma_h2(x0.y, kv.y, a0);
          a0 = fma_h2(x0.z, kv.z, a0);
          a0 = fma_h2(x0.w, kv.w, a0);
          a1 = fma_h2(x1.x, kv.x, a1);
          a1 = fma_h2(x1.y, kv.y, a1);
          a1 = fma_h2(x1.z, kv.z, a1);
          a1 = fma_h2(x1.w, kv.w, a1);
        }
        // the key's dot: (a_q0 + a_q1) + (a_q2 + a_q3)
        a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 8));
        a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 8));
        a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 16));
        a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 16));
        if (valid) {
          s0 = __fmul_rn(a0, kAttnScale);
          s1 = __fmul_rn(a1, kAttnScale);
        }
      }
      const float cm0 = warp_max_redux(s0), cm1 = warp_max_redux(s1);
      float p0 = valid ? q3_expf(__fsub_rn(s0, cm0)) : 0.0f;
      float p1 = valid ? q3_expf(__fsub_rn(s1, cm1)) : 0.0f;
      // chunk sums over the 8 keys: ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7))
      float cl0 = p0, cl1 = p1;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        cl0 = __fadd_rn(cl0, __shfl_xor_sync(0xffffffffu, cl0, off));
        cl1 = __fadd_rn(cl1, __shfl_xor_sync(0xffffffffu, cl1, off));
      }
      if (j == 0) fphase(a.phase, 8);
      // p.v: lane = dims 4 lane .. 4 lane + 3, keys in order (p of key tt from lane tt);
      // keys past the end have p = 0 and V = 0 and add an exact +0
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int tt = 0; tt < kFaChunk; ++tt) {
        const float pa = __shfl_sync(0xffffffffu, p0, tt), pb = __shfl_sync(0xffffffffu, p1, tt);
        const int64_t tk = t0 + tt;
        uint2 vt = make_uint2(0u, 0u);
        if (tk < pos)
          asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];"
                       : "=r"(vt.x), "=r"(vt.y) : "r"(slot + kFaKTile + tt * kHD * 2 + 8 * lane));
        else if (tk == pos)
          vt = *reinterpret_cast<const uint2*>(qkv_h + 3 * kHD + 4 * lane);
        const float v0 = h2f((uint16_t)(vt.x & 0xffffu)), v1 = h2f((uint16_t)(vt.x >> 16));
        const float v2 = h2f((uint16_t)(vt.y & 0xffffu)), v3 = h2f((uint16_t)(vt.y >> 16));
        c0[0] = __fmaf_rn(pa, v0, c0[0]);
        c0[1] = __fmaf_rn(pa, v1, c0[1]);
        c0[2] = __fmaf_rn(pa, v2, c0[2]);
        c0[3] = __fmaf_rn(pa, v3, c0[3]);
        c1[0] = __fmaf_rn(pb, v0, c1[0]);
        c1[1] = __fmaf_rn(pb, v1, c1[1]);
        c1[2] = __fmaf_rn(pb, v2, c1[2]);
        c1[3] = __fmaf_rn(pb, v3, c1[3]);
      }
      __syncwarp();  // every lane is done with the slot
      if (j + kFaAttWarps < nloc) issue_chunk(warp, j + kFaAttWarps);
      if (pass == 0) {
        m0 = cm0, l0 = cl0, m1 = cm1, l1 = cl1;
#pragma unroll
        for (int e = 0; e < 4; ++e) o0[e] = c0[e], o1[e] = c1[e];
      } else {
        att_merge(m0, l0, o0, cm0, cl0, c0);
        att_merge(m1, l1, o1, cm1, cl1, c1);
      }
    }
    if (lane == 0) {
      part[warp][0].m = m0, part[warp][0].l = l0;
      part[warp][1].m = m1, part[warp][1].l = l1;
    }
    *reinterpret_cast<float4*>(&part[warp][0].o[4 * lane]) = make_float4(o0[0], o0[1], o0[2], o0[3]);
    *reinterpret_cast<float4*>(&part[warp][1].o[4 * lane]) = make_float4(o1[0], o1[1], o1[2], o1[3]);
  }
  __syncthreads();
  fphase(a.phase, 9);
  // 9) this rank's fold over its 8 warps: thread (head hh, dim d); a warp
  //    without chunks holds m = -inf, l = 0, o = 0
  {
    const int hh = tid >> 7, d = tid & (kHD - 1);
    float M = -__int_as_float(0x7f800000);
#pragma unroll
    for (int w = 0; w < kFaAttWarps; ++w) M = fmaxf(M, part[w][hh].m);
    float l = 0.0f, o = 0.0f;
#pragma unroll
    for (int w = 0; w < kFaAttWarps; ++w) {
      // exp(-inf - M) = 0 leaves l and o unchanged; a rank without chunks
      // (M = -inf) keeps l = o = 0
      const float e = M == -__int_as_float(0x7f800000) ? 0.0f : q3_expf(__fsub_rn(part[w][hh].m, M));
      l = __fmaf_rn(part[w][hh].l, e, l);
      o = __fmaf_rn(part[w][hh].o[d], e, o);
    }
    cpart[hh].o[d] = o;
    if (d == 0) cpart[hh].m = M, cpart[hh].l = l;
  }
  __syncthreads();
  // push (M, l) and 16 dims of o to the rank that folds those dims: rank q
  // owns dims 16q .. 16q+15 of the pair (head q / 8)
  if (tid < 5 * kFC) {
    const int dst = tid / 5, piece = tid % 5, hh = dst >> 3, d0 = 16 * (dst & 7);
    uint4 v;
    if (piece == 0)
      v = make_uint4(__float_as_uint(cpart[hh].m), __float_as_uint(cpart[hh].l), 0u, 0u);
    else
      v = *reinterpret_cast<const uint4*>(&cpart[hh].o[d0 + 4 * (piece - 1)]);
    st_async_v4(smem_u32(&fin[r][4 * piece]), (uint32_t)dst, v, smem_u32(&fbar));
  }
  // 10) fold dims 16r .. 16r+15 over the ranks (lane q < 16 holds rank q's
  //    weight) and push them into every rank's attention output
  if (warp == 0) {
    ok = mbar_wait_own(&fbar, 0u, a.err, kErrTimeoutFull) && ok;
    fphase(a.phase, 10);
    const int q = lane & (kFC - 1);
    const float Mq = fin[q][0];
    const float M = warp_max(lane < kFC ? Mq : -__int_as_float(0x7f800000));
    const float E = q3_expf(__fsub_rn(Mq, M));
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int k = 0; k < kFC; ++k) {
      const float Ek = __shfl_sync(0xffffffffu, E, k);
      L = __fmaf_rn(fin[k][1], Ek, L);
      O = __fmaf_rn(fin[k][4 + q], Ek, O);
    }
    if (lane < kFC) fout[lane] = f2h(__fdiv_rn(O, L));
    __syncwarp();
    const int dst = lane >> 1, piece = lane & 1;
    const uint4 v = reinterpret_cast<const uint4*>(fout)[piece];
    st_async_v4(smem_u32(att + xh_index(kFC * r + 8 * piece)), (uint32_t)dst, v, smem_u32(&abar));
  }
  ok = mbar_wait_own(&abar, 0u, a.err, kErrTimeoutFull) && ok;
  fphase(a.phase, 12);
  const bool ook = mbar_wait_own(&obar, 0u, a.err, kErrTimeoutFull);
  // 11) the head pair's slice of W_o: rows 64r + 8w + i, lane = 4 i + sub takes
  //    blocks 2 sub, 2 sub + 1 (acc = fma(scale, inner, acc) per block), then
  //    v += shfl_xor(v, 1); v += shfl_xor(v, 2)
  {
    const int i = lane >> 2, sub = lane & 3;
    const int row = 8 * warp + i;
    const uint32_t rb = smem_u32(wo) + row * kFaOBytes;
    float acc = 0.0f;
#pragma unroll
    for (int bb = 0; bb < 2; ++bb) {
      const int b = 2 * sub + bb;
      uint32_t xb[16];
      load_xblock(att, b, xb);
      acc = q8_block_dot_mlir(q8_load_block(rb + kQBytes * b), xb, acc);
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    if (sub == 0) a.opart[h * kDim + kFaORows * r + row] = acc;
  }
  // a CTA leaves only with its copies and every rank's pushes into it landed
  // (waited again, bounded, after a wait that gave up)
  if (!ok) {
    mbar_wait_own(&cbar, 0u, nullptr, 0);
    mbar_wait_own(&xbar, 0u, nullptr, 0);
    mbar_wait_own(&qbar, 0u, nullptr, 0);
    mbar_wait_own(&fbar, 0u, nullptr, 0);
    mbar_wait_own(&abar, 0u, nullptr, 0);
  }
  if (!wok) mbar_wait_own(&wbar, 0u, nullptr, 0);
  if (!ook) mbar_wait_own(&obar, 0u, nullptr, 0);
  if (!kvok && warp < kFaAttWarps && nloc > warp) {
    const int passes = (nloc - 1 - warp) / kFaAttWarps + 1;
    mbar_wait_own(&kvbar[warp], (uint32_t)((passes - 1) & 1), nullptr, 0);
  }
  fphase(a.phase, 13);
  ktrace_end(a.trace);
}

// ===========================================================================
// k_fused_ffn: grid 8 clusters x 16 CTAs, 384 threads.
// ===========================================================================
// Down order (restated by the oracle): rank r of cluster c produces rows
// 64r .. 64r+63 of dpart[c]; lane = 4 i + sub of warp w (row 64r + 8w + i)
// takes blocks 12c + 3 sub .. 12c + 3 sub + 2 (acc = fma(scale, inner, acc)
// per block), then v += shfl_xor(v, 1); v += shfl_xor(v, 2).
__global__ void __launch_bounds__(kFbThreads, 1) k_fused_ffn(const __grid_constant__ FbArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* wg = smem;
  uint8_t* wu = smem + kFbGUBytes;
  uint8_t* wd = smem + 2 * kFbGUBytes;  // 128-byte aligned (the box destination)
  __shared__ __align__(16) uint16_t hr[kDim];
  __shared__ __align__(16) float4 xss[kFC];
  __shared__ __align__(16) uint16_t yloc[kFSlice];
  __shared__ __align__(16) uint4 ssl;
  __shared__ __align__(16) uint16_t xs[kDim / kQBlk * kXhStride];
  __shared__ __align__(16) uint16_t act_loc[kFbAct];  // 48 bytes: 3 pushes of 8
  __shared__ __align__(16) uint16_t act_all[kFbDBlocks * kXhStride];
  __shared__ __align__(8) uint64_t wbar, dbar, cbar, hbar, actbar;
  __shared__ __align__(16) uint16_t gam[kDim];  // ffn_norm gamma

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x / kFC;
  const int r = (int)cluster_rank();
  ktrace_start(a.trace);
  fphase(a.phase, 0);
  if (tid == 0) {
    mbar_init(&wbar, 1);
    mbar_init(&dbar, 1);
    mbar_init(&cbar, 1);
    mbar_init(&hbar, 1);
    mbar_init(&actbar, 1);
    fence_mbar_init();
    mbar_expect_tx(&hbar, kFSliceBytes);
    mbar_expect_tx(&actbar, kFC * 3 * 16);
  }
  __syncthreads();
  pdl_launch_dependents();
  if (a.stop != nullptr && *a.stop != 0) return;  // uniform over the grid (see k_fused_attn)
  cluster_sync_all();  // every rank's exchange barriers are initialised

  const uint64_t pol_w = l2_policy_evict_first();
  // W_down row window: the slice's 12 blocks start at byte 408c of a row,
  // which is 16-byte aligned for even c and 8 bytes past a boundary for odd c
  const uint32_t dwin0 = (uint32_t)(kFbDBlocks * kQBytes * c) & ~15u;
  const uint32_t dboff = (uint32_t)(kFbDBlocks * kQBytes * c) - dwin0;
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&a.wd_map);
    mbar_expect_tx(&wbar, 2 * kFbGUBytes);
    const int g0 = kFbSlice * c + kFbAct * r;  // first gate row (= act index)
    bulk_g2s(wg, a.wgu + (int64_t)g0 * kRow1K, kFbGUBytes, &wbar, pol_w);
    bulk_g2s(wu, a.wgu + (int64_t)(kFFN + g0) * kRow1K, kFbGUBytes, &wbar, pol_w);
  }
  if (warp == 2 && lane == 0) {  // the gamma by bulk copy (see k_fused_attn)
    mbar_expect_tx(&cbar, kDim * 2);
    bulk_g2s(gam, a.ffn_norm, kDim * 2, &cbar, l2_policy_evict_normal());
  }

  fphase(a.phase, 7);
  pdl_wait();  // x and the O partials are visible
  ktrace_release(a.trace);
  fphase(a.phase, 1);

  // 1) this rank's slice of h1 = f16(x + f16(sum_h opart[h])) (cluster 0
  //    publishes it), pushed with its sum of squares
  if (warp == 0) {
    const int k0 = kFSlice * r + 4 * (lane & 15);
    uint2 hv = make_uint2(0u, 0u);
    if (lane < 16) {
      hv = resid_plus_parts(a.x, a.opart, k0);
      if (c == 0) *reinterpret_cast<uint2*>(a.h1_out + k0) = hv;
    }
    push_slice(hv, r, lane, yloc, hr, xss, &ssl, &hbar);
  }
  bool ok = mbar_wait_own(&hbar, 0u, a.err, kErrTimeoutFull);
  ok = mbar_wait_own(&cbar, 0u, a.err, kErrTimeoutFull) && ok;
  // 2) RMSNorm with ffn_norm
  slice_rmsnorm(hr, xss, gam, xs);
  fphase(a.phase, 2);
  // the W_down window is needed last: its copy goes out now (after the
  // residual slices' L2 round trip)
  if (warp == 1 && lane == 0) {
    mbar_expect_tx(&dbar, kFbDBytes);
    tma_load_2d(wd, &a.wd_map, (int)(dwin0 / 4), a.layer * kDim + kFbDRows * r, &dbar);
  }

  // 3) gate|up rows: warp w -> act values 2w, 2w+1 of this CTA; lane = block
  const bool wok = mbar_wait_own(&wbar, 0u, a.err, kErrTimeoutFull);
  fphase(a.phase, 3);
  {
    // the warp's two gate and two up rows, their chains interleaved (the
    // operations of q8_block_dot_mlir + warp_sum for each row); lanes 0 and
    // 1 apply SwiGLU to the two act values
    uint32_t xb[16];
    load_xblock(xs, lane, xb);
    const int row = 2 * warp;
    const Q8BlockWords bw[4] = {q8_load_block(smem_u32(wg) + row * kRow1K + kQBytes * lane),
                                q8_load_block(smem_u32(wu) + row * kRow1K + kQBytes * lane),
                                q8_load_block(smem_u32(wg) + (row + 1) * kRow1K + kQBytes * lane),
                                q8_load_block(smem_u32(wu) + (row + 1) * kRow1K + kQBytes * lane)};
    float d[4];
    q8_block_dot4_mlir(bw, xb, d);
    warp_sum4(d);
    if (lane < 2)
      act_loc[row + lane] = swiglu_h(f2h(lane == 0 ? d[0] : d[2]), f2h(lane == 0 ? d[1] : d[3]));
  }
  __syncthreads();
  fphase(a.phase, 4);
  // 4) every rank pushes its 24 act values (3 x 8) into every rank's copy of
  //    the slice's 384 (block layout; a group of 8 never crosses a block)
  if (tid < 3 * kFC) {
    const int dst = tid / 3, piece = tid % 3;
    const uint4 v = reinterpret_cast<const uint4*>(act_loc)[piece];
    st_async_v4(smem_u32(act_all + xh_index(kFbAct * r + 8 * piece)), (uint32_t)dst, v,
                smem_u32(&actbar));
  }
  ok = mbar_wait_own(&actbar, 0u, a.err, kErrTimeoutFull) && ok;
  fphase(a.phase, 5);
  const bool dok = mbar_wait_own(&dbar, 0u, a.err, kErrTimeoutFull);
  // 5) the slice's columns of W_down
  if (warp < kFbDRows / 8) {
    const int i = lane >> 2, sub = lane & 3;
    const int row = 8 * warp + i;
    const uint32_t rb = smem_u32(wd) + row * kFbDWin + dboff;
    float acc = 0.0f;
#pragma unroll
    for (int bb = 0; bb < 3; ++bb) {
      const int b = 3 * sub + bb;
      uint32_t xb[16];
      load_xblock(act_all, b, xb);
      acc = q8_block_dot_mlir(q8_load_block(rb + kQBytes * b), xb, acc);
    }
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    if (sub == 0) a.dpart[c * kDim + kFbDRows * r + row] = acc;
  }
  if (a.advance != nullptr && blockIdx.x == 0 && tid == 0) a.advance->pos += 1;
  if (!ok) {
    mbar_wait_own(&cbar, 0u, nullptr, 0);
    mbar_wait_own(&hbar, 0u, nullptr, 0);
    mbar_wait_own(&actbar, 0u, nullptr, 0);
  }
  if (!wok) mbar_wait_own(&wbar, 0u, nullptr, 0);
  if (!dok) mbar_wait_own(&dbar, 0u, nullptr, 0);
  fphase(a.phase, 6);
  ktrace_end(a.trace);
}

// x = f16(res + f16(sum of the kFParts partial vectors)): one CTA of 256
// threads (the stateless layer entry point's last step).
__global__ void __launch_bounds__(256) k_resid_parts(const uint16_t* res, const float* parts,
                                                    uint16_t* out) {
  pdl_wait();
  *reinterpret_cast<uint2*>(out + 4 * threadIdx.x) = resid_plus_parts(res, parts, 4 * threadIdx.x);
}

}  // namespace q3
