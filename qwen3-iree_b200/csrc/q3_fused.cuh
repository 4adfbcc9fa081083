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
constexpr int kFaAttWarps = 2;                       // warps that own a K/V chunk slot
constexpr uint32_t kFaKStride = 272;                 // padded K row: lane-per-key reads conflict-free
constexpr uint32_t kFaKTile = kAttChunk * kFaKStride;  // 8704
constexpr uint32_t kFaVTile = kAttChunk * kHD * 2;     // 8192
constexpr uint32_t kFaSlot = kFaKTile + kFaVTile;
constexpr uint32_t kFaWqkvBytes = kFaRows * kRow1K;          // 34816
constexpr uint32_t kFaWoBytes = kFaORows * kFaOBytes;        // 17408
constexpr uint32_t kFaSmem = kFaWqkvBytes + kFaWoBytes + kFaAttWarps * kFaSlot;  // 86016
constexpr int kFaMaxLocal = 8;  // chunks per CTA: caches up to 8 * 16 * 32 = 4096 positions
constexpr int64_t kFusedMaxPositions = (int64_t)kFaMaxLocal * kFC * kAttChunk;

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
  const uint8_t* wq;          // this layer's W_q [2048, 1024] Q8_0 (reference layout)
  const uint8_t* wk;          // W_k [1024, 1024]
  const uint8_t* wv;          // W_v [1024, 1024]
  const uint8_t* wo;          // W_o [1024, 2048]
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
  const SeqState* seq;
  int* err;
  unsigned long long* trace;  // optional launch timing record
  long long* phase;           // optional per-CTA phase stamps [grid][kFPhases] (ns)
};

struct FbArgs {
  const uint8_t* wgu;         // this layer's W_gate|up [6144, 1024] (gate rows, then up rows)
  const uint8_t* wd;          // W_down [1024, 3072]
  const uint16_t* ffn_norm;   // [1024]
  const uint16_t* x;          // residual (the attention kernel's x_out)
  const float* opart;         // [8][1024]
  uint16_t* h1_out;           // h1, written by CTA 0 (the next layer's residual)
  float* dpart;               // out: [8][1024] down partials (one per FFN slice)
  const SeqState* seq;
  SeqState* advance;          // if set, pos += 1 (the last kernel of a prompt-ingestion step)
  int* err;
  unsigned long long* trace;
  long long* phase;           // optional per-CTA phase stamps [grid][kFPhases] (ns)
};

// Phase stamps (latency analysis): thread 0 of each CTA records %globaltimer
// at the end of each numbered step of the kernels below.
constexpr int kFPhases = 12;
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

// A K = 1024 x block (32 f16) from shared memory in the 40-half block layout.
__device__ __forceinline__ void load_xblock(const uint16_t* xs, int b, uint32_t (&xb)[16]) {
  const uint4* p = reinterpret_cast<const uint4*>(xs + b * kXhStride);
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint4 t = p[v];
    xb[4 * v] = t.x, xb[4 * v + 1] = t.y, xb[4 * v + 2] = t.z, xb[4 * v + 3] = t.w;
  }
}

// x (f16 [1024], xr) -> xs = f16((x / r) * g) in the block layout, r =
// sqrt(ss/1024 + eps) with ss in warp 0's lane-strided fma order + butterfly
// (the exact engine's RMSNorm).  gr[i] = g[threadIdx.x + 256 i] for the first
// 256 threads.  Called by every thread; begins and ends with __syncthreads.
__device__ __forceinline__ void fused_rmsnorm(const uint16_t* xr, const uint16_t (&gr)[4],
                                              uint16_t* xs, float* rs) {
  __syncthreads();
  if (threadIdx.x < 32) {
    float ss = 0.0f;
#pragma unroll 8
    for (int k = threadIdx.x; k < kDim; k += 32) {
      const float v = h2f(xr[k]);
      ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if (threadIdx.x == 0) *rs = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kDim), kEps));
  }
  __syncthreads();
  if (threadIdx.x < 256) {
    const float r = *rs;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int k = threadIdx.x + 256 * i;
      xs[xh_index(k)] = rms_apply(xr[k], gr[i], r);
    }
  }
  __syncthreads();
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
// out_d = f16(O_d / L).  A rank without chunks contributes M_r = -inf.
__global__ void __launch_bounds__(kFaThreads, 1) k_fused_attn(const __grid_constant__ FaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* wqkv = smem;
  uint8_t* wo = smem + kFaWqkvBytes;
  uint8_t* kvs = wo + kFaWoBytes;
  __shared__ __align__(16) uint16_t xr[kDim];
  __shared__ __align__(16) uint16_t xs[kDim / kQBlk * kXhStride];
  __shared__ __align__(16) uint16_t loc[kFaRows];
  __shared__ __align__(16) uint16_t qkv_h[4 * kHD];  // q head 2h | q head 2h+1 | k | v (raw)
  __shared__ __align__(16) uint16_t qs[2][kHD];
  __shared__ __align__(16) uint16_t ks[kHD];
  __shared__ __align__(16) AttnPartial part[kFaMaxLocal][2];
  __shared__ __align__(16) AttnPartial cpart[2];
  __shared__ __align__(16) float2 pw[kFaAttWarps][kAttChunk];
  __shared__ __align__(16) uint16_t att[2 * kHD / kQBlk * kXhStride];
  __shared__ __align__(8) uint64_t wbar, kvbar[kFaAttWarps];
  __shared__ float rs;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x / kFC;
  const int r = (int)cluster_rank();
  ktrace_start(a.trace);
  fphase(a.phase, 0);
  if (tid == 0) {
    mbar_init(&wbar, 1);
    for (int i = 0; i < kFaAttWarps; ++i) mbar_init(&kvbar[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  // The decode state changes only in a step's last kernel, and every step is
  // its own graph launch: read it before the wait.  It is the same for every
  // CTA, so a CTA that returns here takes its whole cluster with it.
  if (a.seq->stop != 0) return;
  const int64_t pos = a.seq->pos;
  if (pos < 0 || pos >= a.S || attn_nchunks(pos) > kFC * kFaMaxLocal) {
    if (tid == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    return;
  }
  const int64_t T = pos + 1;
  const int nch = attn_nchunks(pos);
  const int nloc = r < nch ? (nch - 1 - r) / kFC + 1 : 0;  // local chunks j: ci = r + 16 j

  // ---- bulk copies that do not depend on the previous kernel
  const uint64_t pol_w = l2_policy_evict_first();
  const uint64_t pol_kv = l2_policy_evict_normal();
  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(&wbar, kFaWqkvBytes + kFaWoBytes);
      bulk_g2s(wqkv, a.wq + (int64_t)(2 * kHD * h + kFaQRows * r) * kRow1K, kFaQRows * kRow1K,
               &wbar, pol_w);
      bulk_g2s(wqkv + kFaQRows * kRow1K, a.wk + (int64_t)(kHD * h + kFaKRows * r) * kRow1K,
               kFaKRows * kRow1K, &wbar, pol_w);
      bulk_g2s(wqkv + (kFaQRows + kFaKRows) * kRow1K,
               a.wv + (int64_t)(kHD * h + kFaKRows * r) * kRow1K, kFaKRows * kRow1K, &wbar, pol_w);
    }
    __syncwarp();
    for (int i = lane; i < kFaORows; i += 32)
      bulk_g2s(wo + i * kFaOBytes, a.wo + (int64_t)(kFaORows * r + i) * kORowBytes + kFaOBytes * h,
               kFaOBytes, &wbar, pol_w);
  }
  // cached keys (< pos) of local chunk j into warp w's slot; the whole warp calls
  auto issue_chunk = [&](int w, int j) {
    const int64_t t0 = (int64_t)(r + kFC * j) * kAttChunk;
    int64_t nk = pos - t0;
    nk = nk < 0 ? 0 : (nk > kAttChunk ? kAttChunk : nk);
    uint8_t* slot = kvs + w * kFaSlot;
    if (lane == 0) mbar_expect_tx(&kvbar[w], (uint32_t)nk * 2u * kHD * 2u);
    __syncwarp();
    if (lane < nk) {
      const int64_t off = (a.slot0 + t0 + lane) * (kNKV * kHD) + h * kHD;
      bulk_g2s(slot + lane * kFaKStride, a.kc + off, kHD * 2, &kvbar[w], pol_kv);
      bulk_g2s(slot + kFaKTile + lane * kHD * 2, a.vc + off, kHD * 2, &kvbar[w], pol_kv);
    }
  };
  if (warp < kFaAttWarps && warp < nloc) issue_chunk(warp, warp);

  // constants: gammas, RoPE angles at pos, the layer-0 embedding row
  uint16_t gr[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) gr[i] = a.attn_norm[tid + 256 * i];
  float rc0 = 0.f, rs0 = 0.f, rc1 = 0.f, rs1 = 0.f;
  uint16_t gv[4] = {0, 0, 0, 0};
  if (warp < 3) {
    const float* ct = a.rope_cos + pos * 64;
    const float* sn = a.rope_sin + pos * 64;
    rc0 = ct[lane], rs0 = sn[lane], rc1 = ct[lane + 32], rs1 = sn[lane + 32];
    const uint16_t* g = warp < 2 ? a.q_norm : a.k_norm;
#pragma unroll
    for (int i = 0; i < 4; ++i) gv[i] = g[lane + 32 * i];
  }
  uint2 xemb = make_uint2(0u, 0u);
  if (a.tokens != nullptr) {
    int64_t tok = a.tokens[pos];
    if (tok < 0 || tok >= kVocab) {
      if (tid == 0 && a.err) atomicCAS(a.err, 0, kErrBadToken);
      tok = 0;
    }
    xemb = *reinterpret_cast<const uint2*>(a.embd + tok * (int64_t)kDim + 4 * tid);
  }

  pdl_wait();  // the previous kernel's outputs (h1, dpart) are visible
  ktrace_release(a.trace);
  fphase(a.phase, 1);

  // 1) the residual stream x (4 values per thread); CTA 0 publishes it
  {
    const uint2 xv = a.tokens != nullptr ? xemb
                     : a.dpart == nullptr ? __ldcg(reinterpret_cast<const uint2*>(a.h1 + 4 * tid))
                                          : resid_plus_parts(a.h1, a.dpart, 4 * tid);
    *reinterpret_cast<uint2*>(xr + 4 * tid) = xv;
    if (blockIdx.x == 0) *reinterpret_cast<uint2*>(a.x_out + 4 * tid) = xv;
  }
  // 2) RMSNorm with attn_norm
  fused_rmsnorm(xr, gr, xs, &rs);
  fphase(a.phase, 2);

  // 3) Q|K|V rows: warp w takes rows w, w+8 (q), w+16 (k), w+24 (v); lane = block
  const bool wok = mbar_wait_own(&wbar, 0u, a.err, kErrTimeoutFull);
  fphase(a.phase, 3);
  {
    uint32_t xb[16];
    load_xblock(xs, lane, xb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = warp + 8 * i;
      const Q8BlockWords bw = q8_load_block(smem_u32(wqkv) + row * kRow1K + kQBytes * lane);
      const float d = warp_sum(q8_block_dot_mlir(bw, xb, 0.0f));
      if (lane == 0) loc[row] = f2h(d);
    }
  }
  cluster_sync_all();  // every rank's Q|K|V rows are visible to the cluster
  fphase(a.phase, 4);

  // 4) the head pair's raw q (2 x 128), k and v from the 16 ranks
  {
    qkv_h[tid] = ld_dsmem_u16(smem_u32(&loc[tid % kFaQRows]), (uint32_t)(tid / kFaQRows));
    if (tid < kHD) {
      const uint32_t src = (uint32_t)(tid / kFaKRows);
      qkv_h[2 * kHD + tid] = ld_dsmem_u16(smem_u32(&loc[kFaQRows + tid % kFaKRows]), src);
      qkv_h[3 * kHD + tid] = ld_dsmem_u16(smem_u32(&loc[kFaQRows + kFaKRows + tid % kFaKRows]), src);
    }
  }
  __syncthreads();
  // 5) QK-norm + RoPE: q heads by warps 0, 1; the k head by warp 2
  if (warp < 3)
    head_norm_rope_smem(qkv_h + (warp < 2 ? warp : 2) * kHD, gv, rc0, rs0, rc1, rs1, lane,
                        warp < 2 ? qs[warp] : ks);
  __syncthreads();
  fphase(a.phase, 5);
  // the new K (normed, roped) and V (raw) rows at slot layer*S + pos
  if (r == 0 && tid < kHD) {
    const int64_t off = (a.slot0 + pos) * (kNKV * kHD) + h * kHD + tid;
    a.kc[off] = ks[tid];
    a.vc[off] = qkv_h[3 * kHD + tid];
  }

  // 6) this rank's chunks: warp w < 2 takes local chunks w, w+2, ... through its slot
  bool kvok = true;
  if (warp < kFaAttWarps) {
    const uint8_t* slot = kvs + warp * kFaSlot;
    int pass = 0;
    for (int j = warp; j < nloc; j += kFaAttWarps, ++pass) {
      kvok = mbar_wait_own(&kvbar[warp], (uint32_t)(pass & 1), a.err, kErrTimeoutFull) && kvok;
      const int64_t t0 = (int64_t)(r + kFC * j) * kAttChunk;
      const int64_t t = t0 + lane;
      const bool valid = t < T;
      float s0 = -__int_as_float(0x7f800000), s1 = s0;
      if (valid) {
        const uint4* kr = t == pos ? reinterpret_cast<const uint4*>(ks)
                                   : reinterpret_cast<const uint4*>(slot + lane * kFaKStride);
        const uint4* q0 = reinterpret_cast<const uint4*>(qs[0]);
        const uint4* q1 = reinterpret_cast<const uint4*>(qs[1]);
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int v = 0; v < kHD / 8; ++v) {
          const uint4 kv = kr[v], x0 = q0[v], x1 = q1[v];
          a0 = fma_h2(x0.x, kv.x, a0);
          a0 = fma_h2(x0.y, kv.y, a0);
          a0 = fma_h2(x0.z, kv.z, a0);
          a0 = fma_h2(x0.w, kv.w, a0);
          a1 = fma_h2(x1.x, kv.x, a1);
          a1 = fma_h2(x1.y, kv.y, a1);
          a1 = fma_h2(x1.z, kv.z, a1);
          a1 = fma_h2(x1.w, kv.w, a1);
        }
        s0 = __fmul_rn(a0, kAttnScale);
        s1 = __fmul_rn(a1, kAttnScale);
      }
      const float m0 = warp_max_redux(s0), m1 = warp_max_redux(s1);
      const float p0 = valid ? q3_expf(__fsub_rn(s0, m0)) : 0.0f;
      const float p1 = valid ? q3_expf(__fsub_rn(s1, m1)) : 0.0f;
      const float l0 = warp_sum(p0), l1 = warp_sum(p1);
      pw[warp][lane] = make_float2(p0, p1);
      __syncwarp();
      // p.v: lane = head dims 4 lane .. 4 lane + 3, keys in order; keys past
      // the end have p = 0 and V = 0 and add an exact +0
      float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
      for (int tt = 0; tt < kAttChunk; ++tt) {
        const float2 pp = pw[warp][tt];
        const int64_t tk = t0 + tt;
        uint2 vt = make_uint2(0u, 0u);
        if (tk < pos)
          vt = *reinterpret_cast<const uint2*>(slot + kFaKTile + tt * kHD * 2 + 8 * lane);
        else if (tk == pos)
          vt = *reinterpret_cast<const uint2*>(qkv_h + 3 * kHD + 4 * lane);
        const float v0 = h2f((uint16_t)(vt.x & 0xffffu)), v1 = h2f((uint16_t)(vt.x >> 16));
        const float v2 = h2f((uint16_t)(vt.y & 0xffffu)), v3 = h2f((uint16_t)(vt.y >> 16));
        o0[0] = __fmaf_rn(pp.x, v0, o0[0]);
        o0[1] = __fmaf_rn(pp.x, v1, o0[1]);
        o0[2] = __fmaf_rn(pp.x, v2, o0[2]);
        o0[3] = __fmaf_rn(pp.x, v3, o0[3]);
        o1[0] = __fmaf_rn(pp.y, v0, o1[0]);
        o1[1] = __fmaf_rn(pp.y, v1, o1[1]);
        o1[2] = __fmaf_rn(pp.y, v2, o1[2]);
        o1[3] = __fmaf_rn(pp.y, v3, o1[3]);
      }
      if (lane == 0) {
        part[j][0].m = m0, part[j][0].l = l0;
        part[j][1].m = m1, part[j][1].l = l1;
      }
      *reinterpret_cast<float4*>(&part[j][0].o[4 * lane]) = make_float4(o0[0], o0[1], o0[2], o0[3]);
      *reinterpret_cast<float4*>(&part[j][1].o[4 * lane]) = make_float4(o1[0], o1[1], o1[2], o1[3]);
      __syncwarp();  // every lane is done with the slot and with pw
      if (j + kFaAttWarps < nloc) issue_chunk(warp, j + kFaAttWarps);
    }
  }
  __syncthreads();
  fphase(a.phase, 6);
  // 7) this rank's fold: thread (head hh, dim d)
  {
    const int hh = tid >> 7, d = tid & (kHD - 1);
    float M = -__int_as_float(0x7f800000);
    for (int j = 0; j < nloc; ++j) M = fmaxf(M, part[j][hh].m);
    float l = 0.0f, o = 0.0f;
    for (int j = 0; j < nloc; ++j) {
      const float e = q3_expf(__fsub_rn(part[j][hh].m, M));
      l = __fmaf_rn(part[j][hh].l, e, l);
      o = __fmaf_rn(part[j][hh].o[d], e, o);
    }
    cpart[hh].o[d] = o;
    if (d == 0) cpart[hh].m = M, cpart[hh].l = l;
  }
  cluster_sync_all();  // every rank's fold is visible to the cluster
  fphase(a.phase, 7);
  // 8) the cluster's fold; warps 0-3 head 2h, warps 4-7 head 2h+1
  {
    const int hh = warp >> 2, d = tid & (kHD - 1);
    float Mr = -__int_as_float(0x7f800000), lr = 0.0f;
    if (lane < kFC) {
      Mr = ld_dsmem_f32(smem_u32(&cpart[hh].m), (uint32_t)lane);
      lr = ld_dsmem_f32(smem_u32(&cpart[hh].l), (uint32_t)lane);
    }
    float orr[kFC];
#pragma unroll
    for (int q = 0; q < kFC; ++q) orr[q] = ld_dsmem_f32(smem_u32(&cpart[hh].o[d]), (uint32_t)q);
    const float M = warp_max(Mr);
    const float E = lane < kFC ? q3_expf(__fsub_rn(Mr, M)) : 0.0f;
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int q = 0; q < kFC; ++q) {
      const float Eq = __shfl_sync(0xffffffffu, E, q);
      L = __fmaf_rn(__shfl_sync(0xffffffffu, lr, q), Eq, L);
      O = __fmaf_rn(orr[q], Eq, O);
    }
    att[xh_index(hh * kHD + d)] = f2h(__fdiv_rn(O, L));
  }
  cluster_arrive();  // done reading the cluster's shared memory (waited on before exit)
  __syncthreads();
  fphase(a.phase, 8);
  // 9) the head pair's slice of W_o: rows 64r + 8w + i, lane = 4 i + sub takes
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
  // a CTA leaves only with its copies landed and after every rank's DSMEM reads
  if (!wok) mbar_wait_own(&wbar, 0u, nullptr, 0);
  if (!kvok && warp < kFaAttWarps && nloc > warp) {
    const int passes = (nloc - 1 - warp) / kFaAttWarps + 1;
    mbar_wait_own(&kvbar[warp], (uint32_t)((passes - 1) & 1), nullptr, 0);
  }
  fphase(a.phase, 9);
  cluster_wait();
  fphase(a.phase, 10);
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
  uint8_t* wd = smem + 2 * kFbGUBytes;
  __shared__ __align__(16) uint16_t hr[kDim];
  __shared__ __align__(16) uint16_t xs[kDim / kQBlk * kXhStride];
  __shared__ __align__(16) uint16_t act_loc[kFbAct];
  __shared__ __align__(16) uint16_t act_all[kFbDBlocks * kXhStride];
  __shared__ __align__(8) uint64_t wbar;
  __shared__ float rs;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x / kFC;
  const int r = (int)cluster_rank();
  ktrace_start(a.trace);
  fphase(a.phase, 0);
  if (tid == 0) {
    mbar_init(&wbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  if (a.seq->stop != 0) return;  // uniform over the grid (see k_fused_attn)

  const uint64_t pol_w = l2_policy_evict_first();
  // W_down row window: the slice's 12 blocks start at byte 408c of a row,
  // which is 16-byte aligned for even c and 8 bytes past a boundary for odd c
  const uint32_t dwin0 = (uint32_t)(kFbDBlocks * kQBytes * c) & ~15u;
  const uint32_t dboff = (uint32_t)(kFbDBlocks * kQBytes * c) - dwin0;
  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(&wbar, kFbSmem);
      const int g0 = kFbSlice * c + kFbAct * r;  // first gate row (= act index)
      bulk_g2s(wg, a.wgu + (int64_t)g0 * kRow1K, kFbGUBytes, &wbar, pol_w);
      bulk_g2s(wu, a.wgu + (int64_t)(kFFN + g0) * kRow1K, kFbGUBytes, &wbar, pol_w);
    }
    __syncwarp();
    for (int i = lane; i < kFbDRows; i += 32)
      bulk_g2s(wd + i * kFbDWin, a.wd + (int64_t)(kFbDRows * r + i) * kDRowBytes + dwin0, kFbDWin,
               &wbar, pol_w);
  }
  uint16_t gr[4] = {0, 0, 0, 0};
  if (tid < 256) {
#pragma unroll
    for (int i = 0; i < 4; ++i) gr[i] = a.ffn_norm[tid + 256 * i];
  }

  pdl_wait();  // x and the O partials are visible
  ktrace_release(a.trace);
  fphase(a.phase, 1);

  // 1) h1 = f16(x + f16(sum_h opart[h])); CTA 0 publishes it
  if (tid < 256) {
    const uint2 hv = resid_plus_parts(a.x, a.opart, 4 * tid);
    *reinterpret_cast<uint2*>(hr + 4 * tid) = hv;
    if (blockIdx.x == 0) *reinterpret_cast<uint2*>(a.h1_out + 4 * tid) = hv;
  }
  // 2) RMSNorm with ffn_norm
  fused_rmsnorm(hr, gr, xs, &rs);
  fphase(a.phase, 2);

  // 3) gate|up rows: warp w -> act values 2w, 2w+1 of this CTA; lane = block
  const bool wok = mbar_wait_own(&wbar, 0u, a.err, kErrTimeoutFull);
  fphase(a.phase, 3);
  {
    uint32_t xb[16];
    load_xblock(xs, lane, xb);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int row = 2 * warp + i;
      const float g = warp_sum(q8_block_dot_mlir(
          q8_load_block(smem_u32(wg) + row * kRow1K + kQBytes * lane), xb, 0.0f));
      const float u = warp_sum(q8_block_dot_mlir(
          q8_load_block(smem_u32(wu) + row * kRow1K + kQBytes * lane), xb, 0.0f));
      if (lane == 0) act_loc[row] = swiglu_h(f2h(g), f2h(u));
    }
  }
  cluster_sync_all();  // every rank's act values are visible to the cluster
  fphase(a.phase, 4);
  // 4) the slice's 384 act values from the 16 ranks
  act_all[xh_index(tid)] = ld_dsmem_u16(smem_u32(&act_loc[tid % kFbAct]), (uint32_t)(tid / kFbAct));
  cluster_arrive();  // done reading the cluster's shared memory (waited on before exit)
  __syncthreads();
  fphase(a.phase, 5);
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
  if (!wok) mbar_wait_own(&wbar, 0u, nullptr, 0);
  fphase(a.phase, 6);
  cluster_wait();
  fphase(a.phase, 7);
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
