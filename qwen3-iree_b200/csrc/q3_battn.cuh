// q3_battn.cuh -- decode attention for the batched decoder (sm_100a).
//
// Same operation as q3_attn.cuh -- QK-RMSNorm (model/qwen3_full.mlir:646-702),
// RoPE (:324-454), the KV write at slot layer*S + pos (:793-797) and GQA
// attention over keys 0..pos (:456-530) -- for B sequences with their own
// positions, built for HBM throughput instead of batch-1 latency:
//
//   * CTA = (kv head h, segment of 512 keys, sequence b); a producer thread
//     streams 32-key K and V tiles (one 8 KB tensor-TMA box each, the cache
//     seen as [B*28*S rows, 1024] f16) through a ring of stages.  Cache rows
//     below pos were written by earlier launches, so the stream starts before
//     the wait on the previous kernel; only q and the new row need it.
//   * 4 consumer warps take chunks round robin and keep an online softmax
//     (m, l, o) for both q heads of the kv head: lane = key for q.k (each lane
//     reads its K row in a lane-rotated 16-byte order, so a quarter warp hits
//     8 distinct bank groups), lane = 4 head dims for p.v.
//   * the warps' states merge in warp order; a sequence whose keys span
//     several segments publishes one partial per segment and the CTA that
//     finishes last for (b, h) merges them in segment order.
//
// The accumulation order differs from the batch-1 kernel's, so this path is
// held to a tolerance (rel-L2 <= 1e-3), like the rest of the batched decoder.
#pragma once

#include <cuda.h>

#include "q3_attn.cuh"
#include "q3_common.cuh"
#include "q3_tc.cuh"

namespace q3 {

constexpr int kBaWarps = 4;                       // consumer warps
constexpr int kBaThreads = 32 * (kBaWarps + 1);   // + the producer warp
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
constexpr int kBaSegChunks = 16;                  // default 32-key chunks per CTA (512 keys)
constexpr uint32_t kBaTileBytes = 32u * kHD * 2u; // one 32-key K (or V) tile

struct BAttnArgs {
  CUtensorMap kmap;        // K cache f16 [B*28*S rows, 1024], box {128, 32}
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
  int layer;
  const int64_t* pos;      // pos[b * pos_stride]
  int pos_stride;
  uint16_t* out;           // [npad][2048]
  AttnPartial* part;       // [B][8][max_segs][2]
  unsigned int* counters;  // [B][8]
  int max_segs;
  int seg_chunks;          // 32-key chunks per CTA
  int* err;
  int tag;
  unsigned long long* trace;  // optional launch timing record
};

struct BAttnSmem {
  uint64_t full[kBaFullBars], empty[kBaStages];
  float wm[kBaWarps][2], wl[kBaWarps][2];
  float wo[kBaWarps][2][kHD];
  uint16_t qs[2][kHD];
  uint16_t ks[kHD];
  int last;
};

__host__ __device__ constexpr size_t battn_smem_bytes() {
  return 1024 + (size_t)kBaStages * 2 * kBaTileBytes;
}

__device__ __forceinline__ int battn_nsegs(int64_t pos, int seg_chunks) {
  const int nch = (int)((pos + kAttChunk) / kAttChunk);
  return (nch + seg_chunks - 1) / seg_chunks;
}

__device__ __forceinline__ void battn_named_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 consumer warps
}

__global__ void __launch_bounds__(kBaThreads) k_battn(const __grid_constant__ BAttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(16) BAttnSmem sm;
  const int h = blockIdx.x, seg = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - smem_u32(smem_raw));

  // positions were set by an earlier graph launch: readable before the wait
  const int64_t pos = a.pos[(int64_t)b * a.pos_stride];
  const bool bad = pos < 0 || pos >= a.S || pos >= a.rope_rows ||
                   battn_nsegs(pos, a.seg_chunks) > a.max_segs;
  if (bad || seg >= battn_nsegs(pos, a.seg_chunks)) {
    pdl_launch_dependents();
    if (bad && seg == 0 && h == 0 && threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    return;
  }
  const int nch_all = (int)((pos + kAttChunk) / kAttChunk);
  const int c0 = seg * a.seg_chunks;
  const int nch = nch_all - c0 < a.seg_chunks ? nch_all - c0 : a.seg_chunks;
  const int nsegs = battn_nsegs(pos, a.seg_chunks);
  const int64_t row0 = ((int64_t)b * kLayers + a.layer) * a.S;  // cache row of slot 0

  ktrace_start(a.trace);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kBaFullBars; ++i) mbar_init(&sm.full[i], 1);
    for (int i = 0; i < kBaStages; ++i) mbar_init(&sm.empty[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kBaWarps) {
    // ------------------------------------------------ producer: K/V tiles
    if (lane == 0) {
      prefetch_tmap(&a.kmap);
      prefetch_tmap(&a.vmap);
      int issued = 0;
      for (int i = 0; i < nch; ++i) {
        const int st = i % kBaStages;
        if (i >= kBaStages &&
            !mbar_wait_own(&sm.empty[st], ((i / kBaStages) - 1) & 1, a.err,
                           kErrTimeoutEmpty | (1 << 4) | ((a.tag & 0xff) << 8), kSpinCycles))
          break;
        uint64_t* const fb = &sm.full[i % kBaFullBars];
        mbar_expect_tx(fb, 2 * kBaTileBytes);
        const int y = (int)(row0 + (int64_t)(c0 + i) * kAttChunk);
        tma_load_2d(gbase + st * 2 * kBaTileBytes, &a.kmap, h * kHD, y, fb);
        tma_load_2d(gbase + st * 2 * kBaTileBytes + kBaTileBytes, &a.vmap, h * kHD, y, fb);
        issued = i + 1;
      }
      // no copy in flight at exit: every chunk before issued - kBaStages was
      // consumed, so only the last kBaStages can still be landing
      for (int i = issued > kBaStages ? issued - kBaStages : 0; i < issued; ++i)
        mbar_wait_own(&sm.full[i % kBaFullBars], (i / kBaFullBars) & 1, a.err,
                      kErrTimeoutFull | (2 << 4) | ((a.tag & 0xff) << 8), kSpinCycles);
    }
    return;  // the producer warp takes no part in the consumers' barriers
  }

  // ------------------------------------------------ consumers (warps 0-3)
  pdl_wait();  // q, k, v come from the previous kernel
  ktrace_release(a.trace);
  const uint16_t* qkv = a.qkv + (int64_t)b * 4096;
  if (warp < 3) {
    const float* ct = a.rope_cos + pos * 64;
    const float* sn = a.rope_sin + pos * 64;
    const float cc0 = ct[lane], s0 = sn[lane], cc1 = ct[lane + 32], s1 = sn[lane + 32];
    if (warp < 2)
      head_norm_rope(qkv + (2 * h + warp) * kHD, a.q_norm, cc0, s0, cc1, s1, lane, sm.qs[warp]);
    else
      head_norm_rope(qkv + 2048 + h * kHD, a.k_norm, cc0, s0, cc1, s1, lane, sm.ks);
  }
  battn_named_sync();
  const bool holds_pos = seg == nsegs - 1;
  if (holds_pos && threadIdx.x < kHD) {  // the new K (normed, roped) and V rows
    const int64_t off = ((int64_t)b * kLayers * a.S + (int64_t)a.layer * a.S + pos) * (kNKV * kHD) +
                        h * kHD + threadIdx.x;
    a.kc[off] = sm.ks[threadIdx.x];
    a.vc[off] = __ldcg(reinterpret_cast<const unsigned short*>(qkv) + 3072 + h * kHD + threadIdx.x);
  }
  // q in registers as f16 pairs: lane-rotated order matches the K reads below
  const uint4* q0p = reinterpret_cast<const uint4*>(sm.qs[0]);
  const uint4* q1p = reinterpret_cast<const uint4*>(sm.qs[1]);
  const uint2 vnew = __ldcg(reinterpret_cast<const uint2*>(qkv + 3072 + h * kHD + 4 * lane));

  float m[2] = {-__int_as_float(0x7f800000), -__int_as_float(0x7f800000)};
  float l[2] = {0.0f, 0.0f};
  float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int i = warp; i < nch; i += kBaWarps) {
    const int st = i % kBaStages;
    if (!mbar_wait_own(&sm.full[i % kBaFullBars], (i / kBaFullBars) & 1, a.err,
                       kErrTimeoutFull | (3 << 4) | ((a.tag & 0xff) << 8), kSpinCycles))
      break;
    const int64_t t0 = (int64_t)(c0 + i) * kAttChunk;
    const int tp = pos < t0 + kAttChunk ? (int)(pos - t0) : -1;  // the new key in this chunk
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
          kk = reinterpret_cast<const uint4*>(sm.ks)[cidx];
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
    float p[2], scale[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float cm = warp_max(s[hh]);
      const float mn = fmaxf(m[hh], cm);
      scale[hh] = q3_expf(__fsub_rn(m[hh], mn));
      p[hh] = lane < nvalid ? q3_expf(__fsub_rn(s[hh], mn)) : 0.0f;
      l[hh] = __fmaf_rn(l[hh], scale[hh], warp_sum(p[hh]));
      m[hh] = mn;
#pragma unroll
      for (int d = 0; d < 4; ++d) o[hh][d] = __fmul_rn(o[hh][d], scale[hh]);
    }
    // p.v, lane = head dims 4*lane .. 4*lane+3; a full chunk without the new
    // key (the common case) runs fully unrolled so its shuffles and loads overlap
    auto pv_step = [&](int tt, uint2 vv) {
      const float p0 = __shfl_sync(0xffffffffu, p[0], tt);
      const float p1 = __shfl_sync(0xffffffffu, p[1], tt);
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
  // the warps' states, merged in warp order by warps 0 (q head 2h) and 1 (2h+1)
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    if (lane == 0) {
      sm.wm[warp][hh] = m[hh];
      sm.wl[warp][hh] = l[hh];
    }
    *reinterpret_cast<float4*>(&sm.wo[warp][hh][4 * lane]) =
        make_float4(o[hh][0], o[hh][1], o[hh][2], o[hh][3]);
  }
  battn_named_sync();
  if (warp >= 2) return;
  const int hh = warp;
  float mm = sm.wm[0][hh], ll = sm.wl[0][hh], oo[4];
  {
    const float4 t4 = *reinterpret_cast<const float4*>(&sm.wo[0][hh][4 * lane]);
    oo[0] = t4.x, oo[1] = t4.y, oo[2] = t4.z, oo[3] = t4.w;
  }
  for (int w = 1; w < kBaWarps; ++w) {
    if (sm.wl[w][hh] == 0.0f) continue;  // a warp without chunks
    const float4 t4 = *reinterpret_cast<const float4*>(&sm.wo[w][hh][4 * lane]);
    const float ob[4] = {t4.x, t4.y, t4.z, t4.w};
    att_merge(mm, ll, oo, sm.wm[w][hh], sm.wl[w][hh], ob);
  }
  if (nsegs > 1) {
    AttnPartial* gp = a.part + (((int64_t)b * kNKV + h) * a.max_segs + seg) * 2 + hh;
    if (lane == 0) {
      gp->m = mm;
      gp->l = ll;
    }
    *reinterpret_cast<float4*>(&gp->o[4 * lane]) = make_float4(oo[0], oo[1], oo[2], oo[3]);
    asm volatile("bar.sync 2, 64;" ::: "memory");  // warps 0 and 1
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(a.counters + b * kNKV + h, 1u);
      sm.last = prev == (unsigned)(nsegs - 1);
      if (sm.last) a.counters[b * kNKV + h] = 0u;
      __threadfence();
    }
    asm volatile("bar.sync 2, 64;" ::: "memory");
    if (!sm.last) {
      ktrace_end(a.trace);
      return;
    }
    const AttnPartial* pb = a.part + (((int64_t)b * kNKV + h) * a.max_segs) * 2 + hh;
    mm = __ldcg(&pb->m);
    ll = __ldcg(&pb->l);
    {
      const float4 t4 = __ldcg(reinterpret_cast<const float4*>(&pb->o[4 * lane]));
      oo[0] = t4.x, oo[1] = t4.y, oo[2] = t4.z, oo[3] = t4.w;
    }
    for (int k0 = 1; k0 < nsegs; k0 += 8) {
      float4 ob4[8];
      float mb[8], lb[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (k0 + u < nsegs) {
          const AttnPartial* q = pb + (int64_t)(k0 + u) * 2;
          ob4[u] = __ldcg(reinterpret_cast<const float4*>(&q->o[4 * lane]));
          mb[u] = __ldcg(&q->m);
          lb[u] = __ldcg(&q->l);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (k0 + u < nsegs) {
          const float ob[4] = {ob4[u].x, ob4[u].y, ob4[u].z, ob4[u].w};
          att_merge(mm, ll, oo, mb[u], lb[u], ob);
        }
      }
    }
  }
  uint16_t* outp = a.out + (int64_t)b * 2048 + (2 * h + hh) * kHD + 4 * lane;
  uint2 pk;
  pk.x = (uint32_t)f2h(__fdiv_rn(oo[0], ll)) | ((uint32_t)f2h(__fdiv_rn(oo[1], ll)) << 16);
  pk.y = (uint32_t)f2h(__fdiv_rn(oo[2], ll)) | ((uint32_t)f2h(__fdiv_rn(oo[3], ll)) << 16);
  *reinterpret_cast<uint2*>(outp) = pk;
  ktrace_end(a.trace);
}

}  // namespace q3
