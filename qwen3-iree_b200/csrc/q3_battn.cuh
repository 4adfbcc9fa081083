// q3_battn.cuh -- decode attention for the batched decoder (sm_100a).
//
// Same operation as q3_attn.cuh -- QK-RMSNorm (model/qwen3_full.mlir:646-702),
// RoPE (:324-454), the KV write at slot layer*S + pos (:793-797) and GQA
// attention over keys 0..pos (:456-530) -- for B sequences with their own
// positions, built for HBM throughput instead of batch-1 latency:
//
//   * the work is the list of 32-key chunks of every (sequence b, kv head h),
//     flattened in (b, h, chunk) order; CTA g of a persistent grid (two per
//     SM) takes a contiguous share of it, so every CTA streams about the same
//     number of bytes whatever the mix of positions (no tail wave).  A share
//     cuts the list into pieces, one per (b, h) it touches, and a piece
//     costs about five chunks beyond its own (measured), so shares are equal
//     in chunks + pieces rather than in chunks alone (BaShares).
//   * a producer thread streams the share's 32-key K and V tiles (one 8 KB
//     tensor-TMA box each) through a ring of stages.  The batched decoder
//     keeps its caches head-major, [B][28][8 heads][S][128], so a piece's
//     tiles are contiguous rows; the reference layout [B][28*S][8][128]
//     (the batch-1 model's cache, read by the prompt prefill) is read as
//     [rows, 1024] with a box of one head's 128 columns.  Cache rows below pos were written by
//     earlier launches, so the stream starts before the wait on the previous
//     kernel; only q and the new row need it.
//   * a q warp stages, per piece, the normed and roped q of both q heads of h
//     and the new K/V row (written to the cache once, by the piece that holds
//     the last chunk) in a ring of piece slots; its loads of one piece are
//     issued together, and the gammas and RoPE rows (which do not depend on
//     the previous kernel) before the wait.
//   * 4 consumer warps take chunks round robin and keep an online softmax
//     (m, l, o) for both q heads: lane = key for q.k (each lane reads its K
//     row in a lane-rotated 16-byte order, so a quarter warp hits 8 distinct
//     bank groups), lane = 4 head dims for p.v.  At the end of a piece the
//     warp that finishes it last merges the 4 states in warp order; a (b, h)
//     that spans CTAs publishes one partial per CTA and the CTA that
//     finishes it last merges them in CTA order (the same bits whatever the
//     timing).
//
// The accumulation order differs from the batch-1 kernel's, so this path is
// held to a tolerance (rel-L2 <= 1e-3), like the rest of the batched decoder.
#pragma once

#include <cuda.h>

#include "q3_attn.cuh"
#include "q3_batch.cuh"
#include "q3_common.cuh"
#include "q3_tc.cuh"

namespace q3 {

constexpr int kBaWarps = 4;                       // consumer warps
constexpr int kBaThreads = 32 * (kBaWarps + 2);   // + the producer and the q warp
constexpr int kBaProducer = kBaWarps;             // warp index of the producer
#ifndef Q3_BA_STAGES
#define Q3_BA_STAGES 6
#endif
constexpr int kBaStages = Q3_BA_STAGES;           // K+V tiles in flight per CTA
// Full barriers, chunk i on full[i % kBaFullBars].  Consumer warps take chunks
// round robin, so with one barrier per stage a warp would wait on phase k of a
// stage whose phase k-1 (another warp's chunk) it never saw: TMA copies land
// in any order, and while phase k-1 is still pending a parity wait for phase
// k reads as complete.  A multiple of the warp count gives every warp its own
// barriers (it saw their previous phases itself), and with at least kBaStages
// of them chunk i - kBaFullBars was consumed, its phase closed, before the
// producer arms chunk i.
constexpr int kBaFullBars = ((kBaStages + kBaWarps - 1) / kBaWarps) * kBaWarps;
static_assert(kBaFullBars % kBaWarps == 0 && kBaFullBars >= kBaStages, "full barrier count");
constexpr uint32_t kBaTileBytes = 32u * kHD * 2u; // one 32-key K (or V) tile
constexpr int kBaCtasPerSm = 2;                   // persistent grid: CTAs per SM
constexpr int kBaQSlots = 4;                      // pieces whose q is staged ahead
constexpr int kBaMaxBatch = 64;

struct BAttnArgs {
  CUtensorMap kmap;        // K cache f16 [B*28*S rows, 1024] or head-major [B*28*8*S rows,
                           // 128], box {128, 32}
  CUtensorMap vmap;        // V cache, same
  const uint16_t* qkv;     // [npad][4096] raw projections (q | k | v)
  const uint16_t* q_norm;  // gamma [128]
  const uint16_t* k_norm;
  const float* rope_cos;   // [rope_rows, 64]
  const float* rope_sin;
  int64_t rope_rows;
  uint16_t* kc;            // caches (for the new row)
  uint16_t* vc;
  int64_t S;               // slots per layer
  int64_t seq_rows;        // cache rows between sequences (28 * S; 0: rows share one cache)
  int head_major;          // caches as [seq][28][8 heads][S][128] (a (b, h) piece streams
                           // contiguous rows) instead of [seq][28 * S][8][128]
  int layer;
  int B;                   // sequences, <= 64
  int prefill;             // rows hold consecutive positions of one sequence whose new K/V
                           // rows an earlier kernel wrote: no pre-wait stream, no new row
  const int64_t* pos;      // pos[b * pos_stride]
  int pos_stride;
  uint16_t* out;           // [npad][2048]
  AttnPartial* part;       // [gridDim.x][2 slots][2 q heads]
  unsigned int* counters;  // [B][8], zero between launches
  int piece_units;         // units a (b, h) piece adds to its share's cost (a chunk is
                           // kBaChunkUnits; BaShares)
  int* err;
  int tag;
  unsigned long long* trace;  // optional launch timing record
  long long* phase;           // optional per-CTA phase stamps [CTAs][kBPhases] (ns)
};

// One (b, h) piece of a CTA's share: chunks [u0, u1) of the flattened list,
// of which (b, h) owns [s0, s1).
struct BaPiece {
  int b, h;
  int u0, u1, s0, s1;
};

struct BAttnSmem {
  uint64_t full[kBaFullBars], empty[kBaStages];
  uint64_t qready[kBaQSlots], qfree[kBaQSlots], wfree[2];
  uint64_t geo;                // gfirst / glast / lofirst written (the q warp, after piece 0)
  int nch[kBaMaxBatch];        // chunks of sequence b (per kv head)
  int pre[kBaMaxBatch + 1];    // pre[b] = 8 * sum of nch below b
  long long pos[kBaMaxBatch];
  int b0, bad, lo, hi;
  int gfirst, glast, lofirst;  // CTAs of the first / last piece's (b, h), share start of gfirst
  unsigned int pcnt[2];        // warps done with the piece in state slot p % 2
  __align__(16) uint16_t q[kBaQSlots][2][kHD];
  __align__(16) uint16_t kn[kBaQSlots][kHD];
  __align__(16) uint16_t vn[kBaQSlots][kHD];
  float wm[2][kBaWarps][2], wl[2][kBaWarps][2];
  __align__(16) float wo[2][kBaWarps][2][kHD];
};

__host__ __device__ constexpr size_t battn_smem_bytes() {
  return 1024 + (size_t)kBaStages * 2 * kBaTileBytes;
}

// Partials a grid of `grid` CTAs may publish, and the workspace they and the
// per-(b, h) counters take.
__host__ __device__ constexpr size_t battn_workspace_bytes(int grid, int B) {
  return sizeof(AttnPartial) * (size_t)grid * 4 + (size_t)B * kNKV * 4;
}

// Shares of equal cost.  A 32-key chunk costs kBaChunkUnits; a (b, h) piece
// adds A units ahead of its first chunk (its q staging, its partial last
// chunk, its merges).  Chunk u starts at unit Cs(u) = kBaChunkUnits u +
// A (8 b + h + 1) for its (b, h); CTA g of G takes the chunks whose start
// unit lies in [g C / G, (g+1) C / G), C = kBaChunkUnits T + 8 B A, so its
// share is contiguous.  A > 0 only while C / G >= kBaChunkUnits + A, which
// puts a chunk start in every interval (consecutive starts are at most
// kBaChunkUnits + A apart): no CTA between two others of a (b, h) is empty.
constexpr long long kBaChunkUnits = 8;
// Measured per-piece cost (B200, B=32 and 64 at contexts of 128-4096): 4-6
// chunks; 40 units = 5 chunks.
constexpr int kBaPieceUnits = 40;

struct BaShares {
  long long T, G, C, A;
  __device__ void init(long long T_, long long grid, int B, long long A_) {
    T = T_;
    G = grid < T ? grid : T;
    A = A_ > 0 ? A_ : 0;
    C = kBaChunkUnits * T + (long long)kNKV * B * A;
    if (C / G < kBaChunkUnits + A) {
      A = 0;
      C = kBaChunkUnits * T;
    }
  }
  // start unit of (b, h)'s first chunk
  __device__ long long unit(const BAttnSmem& sm, int b, int h) const {
    return kBaChunkUnits * (sm.pre[b] + (long long)h * sm.nch[b]) + A * (kNKV * b + h + 1);
  }
};

// floor(n / d) for 0 <= n < 2^53, d > 0: a double quotient, corrected.
__device__ __forceinline__ long long battn_div(long long n, long long d) {
  long long q = (long long)((double)n / (double)d);
  if (q * d > n) --q;
  else if ((q + 1) * d <= n) ++q;
  return q;
}

// First chunk of CTA g's share; warp-collective (every lane returns it).
__device__ long long battn_share_lo(const BaShares& s, const BAttnSmem& sm, int B, long long g,
                                    int lane) {
  if (g <= 0) return 0;
  if (g >= s.G) return s.T;
  const long long t = battn_div(g * s.C + s.G - 1, s.G);  // the share's first unit
  // the last (b, h) whose first chunk starts at or before unit t
  const unsigned m0 = __ballot_sync(0xffffffffu, lane < B && s.unit(sm, lane, 0) <= t);
  const unsigned m1 = __ballot_sync(0xffffffffu, lane + 32 < B && s.unit(sm, lane + 32, 0) <= t);
  if (m0 == 0u) return 0;  // t lies before the first chunk
  const int b = m1 ? 63 - __clz((int)m1) : 31 - __clz((int)m0);
  const int h = 31 - __clz((int)__ballot_sync(0xffffffffu, lane < kNKV && s.unit(sm, b, lane) <= t));
  const long long s0 = sm.pre[b] + (long long)h * sm.nch[b];
  const long long u = s0 + ((t - s.unit(sm, b, h) + kBaChunkUnits - 1) >> 3);  // / kBaChunkUnits
  return u < s0 + sm.nch[b] ? u : s0 + sm.nch[b];
}

// The sequence holding flattened chunk u.
__device__ __forceinline__ int battn_seq_of(const BAttnSmem& sm, int B, long long u) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (sm.pre[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// The CTA whose share holds flattened chunk u.
__device__ int battn_share_of(const BaShares& s, const BAttnSmem& sm, int B, long long u) {
  const int lo = battn_seq_of(sm, B, u);
  const int h = ((int)u - sm.pre[lo]) / sm.nch[lo];
  const long long cs = kBaChunkUnits * u + s.A * (kNKV * lo + h + 1);
  return (int)battn_div(cs * s.G, s.C);
}

// Walks the pieces of share [lo, hi): start with (b0, the h holding lo).
struct BaWalker {
  int b, h, lo, hi;
  __device__ void start(const BAttnSmem& sm, int b_first, int lo_, int hi_) {
    b = b_first;
    lo = lo_;
    hi = hi_;
    h = (lo - sm.pre[b]) / sm.nch[b];
  }
  __device__ bool done(const BAttnSmem& sm) const {
    return b >= kBaMaxBatch || sm.pre[b] + h * sm.nch[b] >= hi;
  }
  __device__ BaPiece get(const BAttnSmem& sm) const {
    BaPiece p;
    p.b = b;
    p.h = h;
    p.s0 = sm.pre[b] + h * sm.nch[b];
    p.s1 = p.s0 + sm.nch[b];
    p.u0 = p.s0 > lo ? p.s0 : lo;
    p.u1 = p.s1 < hi ? p.s1 : hi;
    return p;
  }
  __device__ void next() {
    if (++h == kNKV) {
      h = 0;
      ++b;
    }
  }
};

__device__ __forceinline__ void battn_merge_state(float& m, float& l, float (&o)[4], float mb,
                                                  float lb, const float (&ob)[4]) {
  if (lb == 0.0f) return;  // nothing on that side
  if (l == 0.0f) {
    m = mb;
    l = lb;
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = ob[j];
    return;
  }
  att_merge(m, l, o, mb, lb, ob);
}

__global__ void __launch_bounds__(kBaThreads, kBaCtasPerSm) k_battn(const __grid_constant__ BAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(16) BAttnSmem sm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - smem_u32(smem_raw));
  const int B = a.B;
  ktrace_start(a.trace);
  bphase(a.phase, 0, threadIdx.x == 0);  // start

  // ------------------------------------------------ the work list
  // positions were set by an earlier graph launch: readable before the wait
  if (threadIdx.x == 0) {
    sm.bad = 0;
    sm.pcnt[0] = sm.pcnt[1] = 0u;
  }
  __syncthreads();
  if (threadIdx.x < B) {
    const int64_t pos = a.pos[(int64_t)threadIdx.x * a.pos_stride];
    const bool bad = pos < 0 || pos >= a.S || pos >= a.rope_rows;
    sm.pos[threadIdx.x] = pos;
    sm.nch[threadIdx.x] = bad ? 1 : (int)(pos / kAttChunk) + 1;
    if (bad) sm.bad = 1;
  }
  if (threadIdx.x == 32 * kBaProducer) {
    for (int i = 0; i < kBaFullBars; ++i) mbar_init(&sm.full[i], 1);
    for (int i = 0; i < kBaStages; ++i) mbar_init(&sm.empty[i], 1);
    for (int i = 0; i < kBaQSlots; ++i) {
      mbar_init(&sm.qready[i], 32);
      mbar_init(&sm.qfree[i], 32);
    }
    mbar_init(&sm.wfree[0], 32);
    mbar_init(&sm.wfree[1], 32);
    mbar_init(&sm.geo, 32);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == 0) {  // exclusive prefix of 8 * nch over b (B <= 64: two lanes' worth)
    const int v0 = lane < B ? kNKV * sm.nch[lane] : 0;
    const int v1 = lane + 32 < B ? kNKV * sm.nch[lane + 32] : 0;
    int i0 = v0, i1 = v1;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int t0 = __shfl_up_sync(0xffffffffu, i0, d), t1 = __shfl_up_sync(0xffffffffu, i1, d);
      if (lane >= d) i0 += t0, i1 += t1;
    }
    const int tot0 = __shfl_sync(0xffffffffu, i0, 31);
    sm.pre[lane] = i0 - v0;
    sm.pre[lane + 32] = tot0 + i1 - v1;
    if (lane == 31) sm.pre[kBaMaxBatch] = tot0 + i1;
  }
  __syncthreads();
  BaShares sh;
  sh.init(sm.pre[kBaMaxBatch], gridDim.x, B, a.piece_units);
  const long long T = sh.T, G = sh.G;
  const int g = blockIdx.x;
  if (sm.bad || g >= G) {
    pdl_launch_dependents();
    if (sm.bad && g == 0 && threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    return;
  }
  if (warp < 2) {  // this CTA's share: warp 0 its first chunk, warp 1 its end
    const long long gg = g + warp;
    const int l = sh.A == 0 ? (int)battn_div(gg * T + G - 1, G)  // ceil(g T / G)
                            : (int)battn_share_lo(sh, sm, B, gg, lane);
    if (lane == 0) (warp == 0 ? sm.lo : sm.hi) = l;
    if (warp == 0)  // the sequence holding the first chunk
      for (int bb = lane; bb < B; bb += 32)
        if (sm.pre[bb] <= l && l < sm.pre[bb + 1]) sm.b0 = bb;
  }
  __syncthreads();
  pdl_launch_dependents();
  const int lo = sm.lo, hi = sm.hi;
  const int b_first = sm.b0;
  bphase(a.phase, 1, threadIdx.x == 0);  // work list ready

  if (warp == kBaProducer) {
    // ------------------------------------------------ producer: K/V tiles
    if (lane == 0) {
      prefetch_tmap(&a.kmap);
      prefetch_tmap(&a.vmap);
      if (a.prefill) pdl_wait();  // the rows of this pass come from the previous kernel
      const int n = hi - lo;
      int b = b_first, h = (lo - sm.pre[b]) / sm.nch[b];
      int c = lo - sm.pre[b] - h * sm.nch[b];
      int issued = 0;
      for (int i = 0; i < n; ++i) {
        const int st = i % kBaStages;
        if (i >= kBaStages &&
            !mbar_wait_own(&sm.empty[st], ((i / kBaStages) - 1) & 1, a.err,
                           kErrTimeoutEmpty | (1 << 4) | ((a.tag & 0xff) << 8), kSpinCycles))
          break;
        uint64_t* const fb = &sm.full[i % kBaFullBars];
        mbar_expect_tx(fb, 2 * kBaTileBytes);
        const int x = a.head_major ? 0 : h * kHD;
        const int y = a.head_major
                          ? (int)((((int64_t)b * kLayers + a.layer) * kNKV + h) * a.S + (int64_t)c * kAttChunk)
                          : (int)((int64_t)b * a.seq_rows + (int64_t)a.layer * a.S + (int64_t)c * kAttChunk);
        tma_load_2d(gbase + st * 2 * kBaTileBytes, &a.kmap, x, y, fb);
        tma_load_2d(gbase + st * 2 * kBaTileBytes + kBaTileBytes, &a.vmap, x, y, fb);
        issued = i + 1;
        if (++c == sm.nch[b]) {
          c = 0;
          if (++h == kNKV) {
            h = 0;
            ++b;
          }
        }
      }
      // no copy in flight at exit: every chunk before issued - kBaStages was
      // consumed, so only the last kBaStages can still be landing
      for (int i = issued > kBaStages ? issued - kBaStages : 0; i < issued; ++i)
        mbar_wait_own(&sm.full[i % kBaFullBars], (i / kBaFullBars) & 1, a.err,
                      kErrTimeoutFull | (2 << 4) | ((a.tag & 0xff) << 8), kSpinCycles);
    }
    return;  // the producer warp takes no part in the other warps' barriers
  }

  BaWalker wk;
  wk.start(sm, b_first, lo, hi);

  if (warp > kBaProducer) {
    // ------------------------------------------------ q warp: per-piece q, new K/V row
    uint16_t gq[4], gk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      gq[i] = a.q_norm[lane + 32 * i];
      gk[i] = a.k_norm[lane + 32 * i];
    }
    bool waited = false;
    for (int p = 0; !wk.done(sm); ++p, wk.next()) {
      const BaPiece pc = wk.get(sm);
      const int sl = p % kBaQSlots;
      if (p >= kBaQSlots &&
          !mbar_wait_own(&sm.qfree[sl], ((p / kBaQSlots) - 1) & 1, a.err,
                         kErrTimeoutEmpty | (3 << 4) | ((a.tag & 0xff) << 8), kSpinCycles))
        break;
      // this piece holds the (b, h)'s last chunk: it stages and writes the new row
      const bool holds_pos = pc.s1 <= hi && !a.prefill;
      const int64_t pos = sm.pos[pc.b];
      const float* ct = a.rope_cos + pos * 64;
      const float* sn = a.rope_sin + pos * 64;
      const float cc0 = ct[lane], s0 = sn[lane], cc1 = ct[lane + 32], s1 = sn[lane + 32];
      if (!waited) {
        pdl_wait();  // q, k, v come from the previous kernel
        waited = true;
        bphase(a.phase, 2, lane == 0);  // release
      }
      const unsigned short* qkv =
          reinterpret_cast<const unsigned short*>(a.qkv) + (int64_t)pc.b * 4096;
      float q0[4], q1[4], kn[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        q0[i] = h2f(__ldcg(qkv + 2 * pc.h * kHD + lane + 32 * i));
        q1[i] = h2f(__ldcg(qkv + (2 * pc.h + 1) * kHD + lane + 32 * i));
        kn[i] = holds_pos ? h2f(__ldcg(qkv + 2048 + pc.h * kHD + lane + 32 * i)) : 0.0f;
      }
      const uint2 v = holds_pos ? __ldcg(reinterpret_cast<const uint2*>(qkv + 3072 + pc.h * kHD) + lane)
                                : make_uint2(0u, 0u);
      norm_rope_vals(q0, gq, cc0, s0, cc1, s1, lane, sm.q[sl][0]);
      norm_rope_vals(q1, gq, cc0, s0, cc1, s1, lane, sm.q[sl][1]);
      if (holds_pos) {
        norm_rope_vals(kn, gk, cc0, s0, cc1, s1, lane, sm.kn[sl]);
        *reinterpret_cast<uint2*>(&sm.vn[sl][4 * lane]) = v;
        __syncwarp();
        const int64_t off =
            a.head_major
                ? ((((int64_t)pc.b * kLayers + a.layer) * kNKV + pc.h) * a.S + pos) * kHD
                : ((int64_t)pc.b * a.seq_rows + (int64_t)a.layer * a.S + pos) * (kNKV * kHD) + pc.h * kHD;
        *reinterpret_cast<uint2*>(a.kc + off + 4 * lane) =
            *reinterpret_cast<const uint2*>(&sm.kn[sl][4 * lane]);
        *reinterpret_cast<uint2*>(a.vc + off + 4 * lane) = v;
      }
      mbar_arrive(&sm.qready[sl]);
      if (p == 0) {
        // the CTAs of the (b, h) pairs this share cuts: its first piece's
        // first CTA and that CTA's share start, its last piece's last CTA (the
        // merges wait on geo; computed once piece 0's q is out)
        const int bl = battn_seq_of(sm, B, hi - 1);
        const int hl = (hi - 1 - sm.pre[bl]) / sm.nch[bl];
        const int s1l = sm.pre[bl] + (hl + 1) * sm.nch[bl];
        const int hf = (lo - sm.pre[b_first]) / sm.nch[b_first];
        const int s0f = sm.pre[b_first] + hf * sm.nch[b_first];
        int gf = g, gl = g;
        if (lane == 0 && s0f < lo) gf = battn_share_of(sh, sm, B, s0f);
        if (lane == 1 && s1l > hi) gl = battn_share_of(sh, sm, B, s1l - 1);
        gf = __shfl_sync(0xffffffffu, gf, 0);
        gl = __shfl_sync(0xffffffffu, gl, 1);
        const int lof = gf == g ? lo : (int)battn_share_lo(sh, sm, B, gf, lane);
        if (lane == 0) {
          sm.gfirst = gf;
          sm.glast = gl;
          sm.lofirst = lof;
        }
        __syncwarp();
        mbar_arrive(&sm.geo);
      }
    }
    return;
  }

  // ------------------------------------------------ consumers (warps 0-3)
  for (int p = 0; !wk.done(sm); ++p, wk.next()) {
    const BaPiece pc = wk.get(sm);
    const int sl = p % kBaQSlots, ws = p & 1;
    const bool qok = mbar_wait_own(&sm.qready[sl], (p / kBaQSlots) & 1, a.err,
                                   kErrTimeoutFull | (4 << 4) | ((a.tag & 0xff) << 8), kSpinCycles);
    if (p == 0) {
      ktrace_release(a.trace);
      bphase(a.phase, 3, threadIdx.x == 0);  // first piece's q staged
    }
    if (!qok) break;
    const int64_t pos = sm.pos[pc.b];
    const uint4* q0p = reinterpret_cast<const uint4*>(sm.q[sl][0]);
    const uint4* q1p = reinterpret_cast<const uint4*>(sm.q[sl][1]);
    const uint4* knp = reinterpret_cast<const uint4*>(sm.kn[sl]);
    const uint2 vnew = *reinterpret_cast<const uint2*>(&sm.vn[sl][4 * lane]);
    float m[2] = {-__int_as_float(0x7f800000), -__int_as_float(0x7f800000)};
    float l[2] = {0.0f, 0.0f};
    float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    // chunks i of the share go to warp i % 4 (the full barriers' ownership)
    const int ia = pc.u0 - lo, ib = pc.u1 - lo;
    bool ok = true;
    for (int i = ia + ((warp - ia) % kBaWarps + kBaWarps) % kBaWarps; i < ib; i += kBaWarps) {
      const int st = i % kBaStages;
      if (!mbar_wait_own(&sm.full[i % kBaFullBars], (i / kBaFullBars) & 1, a.err,
                         kErrTimeoutFull | (5 << 4) | ((a.tag & 0xff) << 8), kSpinCycles)) {
        ok = false;
        break;
      }
      const int64_t t0 = (int64_t)(lo + i - pc.s0) * kAttChunk;
      // the new key in this chunk (prefill: already in the cache)
      const int tp = (pos < t0 + kAttChunk && !a.prefill) ? (int)(pos - t0) : -1;
      const int nvalid = (pos + 1 - t0) < kAttChunk ? (int)(pos + 1 - t0) : kAttChunk;
      const uint32_t kt = base + st * 2 * kBaTileBytes, vt = kt + kBaTileBytes;
      // q.k, lane = key
      float s[2] = {-__int_as_float(0x7f800000), -__int_as_float(0x7f800000)};
      if (lane < nvalid) {
        // four independent accumulation chains per head (16 FMAs deep, not 128)
        float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < kHD / 8; ++j) {
          const int cidx = (j + lane) & 15;
          uint4 kk;
          if (lane == tp) {
            kk = knp[cidx];
          } else {
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(kk.x), "=r"(kk.y), "=r"(kk.z), "=r"(kk.w)
                         : "r"(kt + (uint32_t)lane * 256u + (uint32_t)cidx * 16u));
          }
          const uint4 x0 = q0p[cidx], x1 = q1p[cidx];
          a0[0] = fma_h2(x0.x, kk.x, a0[0]);
          a0[1] = fma_h2(x0.y, kk.y, a0[1]);
          a0[2] = fma_h2(x0.z, kk.z, a0[2]);
          a0[3] = fma_h2(x0.w, kk.w, a0[3]);
          a1[0] = fma_h2(x1.x, kk.x, a1[0]);
          a1[1] = fma_h2(x1.y, kk.y, a1[1]);
          a1[2] = fma_h2(x1.z, kk.z, a1[2]);
          a1[3] = fma_h2(x1.w, kk.w, a1[3]);
        }
        s[0] = __fmul_rn(__fadd_rn(__fadd_rn(a0[0], a0[1]), __fadd_rn(a0[2], a0[3])), kAttnScale);
        s[1] = __fmul_rn(__fadd_rn(__fadd_rn(a1[0], a1[1]), __fadd_rn(a1[2], a1[3])), kAttnScale);
      }
      float pr[2], scale[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float cm = warp_max(s[hh]);
        const float mn = fmaxf(m[hh], cm);
        scale[hh] = q3_expf(__fsub_rn(m[hh], mn));
        pr[hh] = lane < nvalid ? q3_expf(__fsub_rn(s[hh], mn)) : 0.0f;
        l[hh] = __fmaf_rn(l[hh], scale[hh], warp_sum(pr[hh]));
        m[hh] = mn;
#pragma unroll
        for (int d = 0; d < 4; ++d) o[hh][d] = __fmul_rn(o[hh][d], scale[hh]);
      }
      // p.v, lane = head dims 4*lane .. 4*lane+3; a full chunk without the new
      // key (the common case) runs fully unrolled so its shuffles and loads overlap
      auto pv_step = [&](int tt, uint2 vv) {
        const float p0 = __shfl_sync(0xffffffffu, pr[0], tt);
        const float p1 = __shfl_sync(0xffffffffu, pr[1], tt);
        const float v0 = h2f((uint16_t)(vv.x & 0xffffu)), v1 = h2f((uint16_t)(vv.x >> 16));
        const float v2 = h2f((uint16_t)(vv.y & 0xffffu)), v3 = h2f((uint16_t)(vv.y >> 16));
        o[0][0] = __fmaf_rn(p0, v0, o[0][0]);
        o[0][1] = __fmaf_rn(p0, v1, o[0][1]);
        o[0][2] = __fmaf_rn(p0, v2, o[0][2]);
        o[0][3] = __fmaf_rn(p0, v3, o[0][3]);
        o[1][0] = __fmaf_rn(p1, v0, o[1][0]);
        o[1][1] = __fmaf_rn(p1, v1, o[1][1]);
        o[1][2] = __fmaf_rn(p1, v2, o[1][2]);
        o[1][3] = __fmaf_rn(p1, v3, o[1][3]);
      };
      auto ld_v = [&](int tt) {
        uint2 vv;
        asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];"
                     : "=r"(vv.x), "=r"(vv.y)
                     : "r"(vt + (uint32_t)tt * 256u + (uint32_t)lane * 8u));
        return vv;
      };
      if (nvalid == kAttChunk && tp < 0) {
#pragma unroll
        for (int tt = 0; tt < kAttChunk; ++tt) pv_step(tt, ld_v(tt));
      } else {
        for (int tt = 0; tt < nvalid; ++tt) pv_step(tt, tt == tp ? vnew : ld_v(tt));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[st]);  // the stage may be refilled
    }
    if (!ok) break;
    // ---- this warp's state of the piece, into state slot p % 2
    if (p >= 2 && !mbar_wait_own(&sm.wfree[ws], ((p >> 1) - 1) & 1, a.err,
                                 kErrTimeoutEmpty | (6 << 4) | ((a.tag & 0xff) << 8), kSpinCycles))
      break;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      if (lane == 0) {
        sm.wm[ws][warp][hh] = m[hh];
        sm.wl[ws][warp][hh] = l[hh];
      }
      *reinterpret_cast<float4*>(&sm.wo[ws][warp][hh][4 * lane]) =
          make_float4(o[hh][0], o[hh][1], o[hh][2], o[hh][3]);
    }
    __threadfence_block();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(&sm.pcnt[ws], 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != kBaWarps - 1) continue;
    // ---- the last warp of the piece merges the 4 states in warp order
    __threadfence_block();
    float mm[2], ll[2], oo[2][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mm[hh] = -__int_as_float(0x7f800000);
      ll[hh] = 0.0f;
      oo[hh][0] = oo[hh][1] = oo[hh][2] = oo[hh][3] = 0.0f;
      for (int w = 0; w < kBaWarps; ++w) {
        const float4 t4 = *reinterpret_cast<const float4*>(&sm.wo[ws][w][hh][4 * lane]);
        const float ob[4] = {t4.x, t4.y, t4.z, t4.w};
        battn_merge_state(mm[hh], ll[hh], oo[hh], sm.wm[ws][w][hh], sm.wl[ws][w][hh], ob);
      }
    }
    if (lane == 0) sm.pcnt[ws] = 0u;
    __syncwarp();
    mbar_arrive(&sm.wfree[ws]);   // the state slot may be rewritten
    mbar_arrive(&sm.qfree[sl]);   // every warp is past this piece's q
    const int bh = pc.b * kNKV + pc.h;
    if (pc.s0 < lo || pc.s1 > hi) {
      // (b, h) spans CTAs: publish this CTA's partial, the last one merges
      const int slot = pc.s0 > lo ? 1 : 0;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        AttnPartial* gp = a.part + ((int64_t)g * 2 + slot) * 2 + hh;
        if (lane == 0) {
          gp->m = mm[hh];
          gp->l = ll[hh];
        }
        *reinterpret_cast<float4*>(&gp->o[4 * lane]) =
            make_float4(oo[hh][0], oo[hh][1], oo[hh][2], oo[hh][3]);
      }
      __threadfence();
      __syncwarp();
      if (!mbar_wait_own(&sm.geo, 0u, a.err,
                         kErrTimeoutFull | (7 << 4) | ((a.tag & 0xff) << 8), kSpinCycles))
        break;
      const int g1 = pc.s0 < lo ? sm.gfirst : g, g2 = pc.s1 > hi ? sm.glast : g;
      unsigned last = 0;
      if (lane == 0) {
        const unsigned prevc = atomicAdd(a.counters + bh, 1u);
        last = prevc == (unsigned)(g2 - g1);
        if (last) a.counters[bh] = 0u;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence();
      const int lo1 = pc.s0 < lo ? sm.lofirst : lo;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        mm[hh] = -__int_as_float(0x7f800000);
        ll[hh] = 0.0f;
        oo[hh][0] = oo[hh][1] = oo[hh][2] = oo[hh][3] = 0.0f;
      }
      for (int gg = g1; gg <= g2; gg += 2) {
        // two CTAs' partials loaded before either is merged (CTA order kept)
        const bool two = gg + 1 <= g2;
        float4 t4[2][2];
        float pm[2][2], pl[2][2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k == 1 && !two) break;
          const int sg = (gg + k == g1 && pc.s0 > lo1) ? 1 : 0;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const AttnPartial* q = a.part + ((int64_t)(gg + k) * 2 + sg) * 2 + hh;
            t4[k][hh] = __ldcg(reinterpret_cast<const float4*>(&q->o[4 * lane]));
            pm[k][hh] = __ldcg(&q->m);
            pl[k][hh] = __ldcg(&q->l);
          }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (k == 1 && !two) break;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float ob[4] = {t4[k][hh].x, t4[k][hh].y, t4[k][hh].z, t4[k][hh].w};
            battn_merge_state(mm[hh], ll[hh], oo[hh], pm[k][hh], pl[k][hh], ob);
          }
        }
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint16_t* outp = a.out + (int64_t)pc.b * 2048 + (2 * pc.h + hh) * kHD + 4 * lane;
      uint2 pk;
      pk.x = (uint32_t)f2h(__fdiv_rn(oo[hh][0], ll[hh])) |
             ((uint32_t)f2h(__fdiv_rn(oo[hh][1], ll[hh])) << 16);
      pk.y = (uint32_t)f2h(__fdiv_rn(oo[hh][2], ll[hh])) |
             ((uint32_t)f2h(__fdiv_rn(oo[hh][3], ll[hh])) << 16);
      *reinterpret_cast<uint2*>(outp) = pk;
    }
  }
  bphase(a.phase, 4, threadIdx.x == 0);  // warp 0 done
  ktrace_end(a.trace);
}

// The new K (QK-RMSNorm + RoPE) and V rows of B rows of qkv at their
// positions, one warp per kv head (prefill passes, before k_battn reads them).
struct BKvArgs {
  const uint16_t* qkv;     // [B][4096]
  const uint16_t* k_norm;  // gamma [128]
  const float* rope_cos;   // [rope_rows, 64]
  const float* rope_sin;
  int64_t rope_rows;
  uint16_t* kc;
  uint16_t* vc;
  int64_t S;
  int64_t seq_rows;        // cache rows between rows' sequences (0: one sequence)
  int layer;
  int B;
  const int64_t* pos;      // pos[b * pos_stride]
  int pos_stride;
  int* err;
  unsigned long long* trace;
};

__global__ void __launch_bounds__(32 * kNKV) k_bkv_write(const __grid_constant__ BKvArgs a) {
  __shared__ __align__(16) uint16_t kn[kNKV][kHD];
  const int b = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  ktrace_start(a.trace);
  pdl_launch_dependents();
  pdl_wait();  // qkv comes from the previous kernel
  ktrace_release(a.trace);
  const int64_t pos = a.pos[(int64_t)b * a.pos_stride];
  if (pos < 0 || pos >= a.S || pos >= a.rope_rows) {
    if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    return;
  }
  const float* ct = a.rope_cos + pos * 64;
  const float* sn = a.rope_sin + pos * 64;
  const uint16_t* qkv = a.qkv + (int64_t)b * 4096;
  head_norm_rope(qkv + 2048 + h * kHD, a.k_norm, ct[lane], sn[lane], ct[lane + 32], sn[lane + 32],
                 lane, kn[h]);
  __syncwarp();
  const int64_t off =
      ((int64_t)b * a.seq_rows + (int64_t)a.layer * a.S + pos) * (kNKV * kHD) + h * kHD + 4 * lane;
  *reinterpret_cast<uint2*>(a.kc + off) = *reinterpret_cast<const uint2*>(&kn[h][4 * lane]);
  *reinterpret_cast<uint2*>(a.vc + off) =
      __ldcg(reinterpret_cast<const uint2*>(qkv + 3072 + h * kHD) + lane);
  ktrace_end(a.trace);
}

}  // namespace q3
