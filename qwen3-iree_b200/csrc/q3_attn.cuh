// q3_attn.cuh -- GQA decode attention for sm_100a (one launch per layer).
//
// Replaces, for one layer and one or more independent sequences:
//   QK-RMSNorm (model/qwen3_full.mlir:646-702), RoPE (:324-454), the KV-cache
//   write at slot layer*S + pos (:793-797) and iree_linalg_ext.attention over
//   keys 0..pos (:456-530), with the reference's whole-slice KV copy
//   (:715-720) removed: the kernel attends straight out of the flat cache.
//
// Split-KV flash decode.  CTA (kv head h, split s, sequence b) owns keys
// [256 s, 256 s + 256); each of its 8 warps takes one chunk of 32 keys
// (lane = key for q.k, lane = 4 head dims for p.v), both q heads 2h, 2h+1
// at once so every K/V row is read once.  Chunk results merge left to right
// inside the CTA; split results merge left to right in the last CTA to
// finish (a counter per (sequence, kv head), no spin-waits).  The CPU oracle
// (q3o_attention) states the same order.
#pragma once

#include "q3_common.cuh"
#include "q3_gemv.cuh"

namespace q3 {

struct AttnPartial {
  float m, l;
  float o[kHD];
};

struct AttnArgs {
  const uint16_t* qkv;      // raw GEMV output [q 2048 | k 1024 | v 1024] (f16), per sequence
  int64_t qkv_stride;       // elements between sequences
  const uint16_t* q_norm;   // gamma [128]
  const uint16_t* k_norm;   // gamma [128]
  const float* rope_cos;    // [rope_pos, 64]
  const float* rope_sin;
  int64_t rope_pos;         // rows in the RoPE tables
  uint16_t* kc;             // flat K cache [slots, 8, 128] of sequence 0
  uint16_t* vc;
  int64_t cache_stride;     // elements between sequences' caches
  int64_t slot0;            // layer * S
  int64_t S;                // slots per layer
  const int64_t* pos;       // device position of sequence b at pos[b * pos_stride]
  int pos_stride;
  const int32_t* stop;      // optional: sequence b skipped when stop[b * stop_stride] != 0
  int stop_stride;
  uint16_t* out;            // [B][2048] f16
  int64_t out_stride;
  AttnPartial* part;        // [B][8][max_splits][2]
  unsigned int* counters;   // [B][8], zero between launches
  int max_splits;
  int* err;
};

// Per-head RMSNorm (f16 out) then NeoX RoPE (f16 out) for one 128-wide head.
// Lane l produces outputs l, l+32, l+64, l+96.
__device__ __forceinline__ void head_norm_rope(const uint16_t* x, const uint16_t* g, float c0,
                                               float s0, float c1, float s1, int lane,
                                               uint16_t* dst) {
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
  for (int i = 0; i < 4; ++i) n[i] = h2f(f2h(__fmul_rn(__fdiv_rn(v[i], r), h2f(g[lane + 32 * i]))));
  // pairs (l, l+64) with angle index l, and (l+32, l+96) with angle index l+32
  dst[lane] = f2h(__fsub_rn(__fmul_rn(n[0], c0), __fmul_rn(n[2], s0)));
  dst[lane + 64] = f2h(__fadd_rn(__fmul_rn(n[0], s0), __fmul_rn(n[2], c0)));
  dst[lane + 32] = f2h(__fsub_rn(__fmul_rn(n[1], c1), __fmul_rn(n[3], s1)));
  dst[lane + 96] = f2h(__fadd_rn(__fmul_rn(n[1], s1), __fmul_rn(n[3], c1)));
}

__device__ __forceinline__ void att_merge(float& m, float& l, float (&o)[4], float mb, float lb,
                                          const float (&ob)[4]) {
  const float mm = fmaxf(m, mb);
  const float ea = q3_expf(__fsub_rn(m, mm));
  const float eb = q3_expf(__fsub_rn(mb, mm));
  l = __fmaf_rn(lb, eb, __fmul_rn(l, ea));
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = __fmaf_rn(ob[j], eb, __fmul_rn(o[j], ea));
  m = mm;
}

__global__ void __launch_bounds__(256) k_attn_decode(const __grid_constant__ AttnArgs a) {
  __shared__ __align__(16) uint16_t qs[2][kHD];
  __shared__ __align__(16) uint16_t ks[kHD];
  __shared__ AttnPartial cp[kAttSplitChunks][2];
  __shared__ int is_last;
  const int h = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (a.stop != nullptr && a.stop[(int64_t)b * a.stop_stride] != 0) return;
  const int64_t pos = a.pos[(int64_t)b * a.pos_stride];
  if (pos < 0 || pos >= a.S || pos >= a.rope_pos) {
    if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    return;
  }
  const int64_t T = pos + 1;
  const int nsplit = (int)((T + kAttSplit - 1) / kAttSplit);
  if (split >= nsplit) return;

  const uint16_t* qkv = a.qkv + (int64_t)b * a.qkv_stride;
  uint16_t* kc = a.kc + (int64_t)b * a.cache_stride;
  uint16_t* vc = a.vc + (int64_t)b * a.cache_stride;
  const float* ct = a.rope_cos + pos * 64;
  const float* sn = a.rope_sin + pos * 64;

  // 1) q heads 2h, 2h+1 and k head h: norm + rope into shared memory
  if (warp < 3) {
    const float c0 = ct[lane], s0 = sn[lane], c1 = ct[lane + 32], s1 = sn[lane + 32];
    if (warp < 2)
      head_norm_rope(qkv + (2 * h + warp) * kHD, a.q_norm, c0, s0, c1, s1, lane, qs[warp]);
    else
      head_norm_rope(qkv + 2048 + h * kHD, a.k_norm, c0, s0, c1, s1, lane, ks);
  }
  __syncthreads();
  // 2) the CTA holding key `pos` writes the new K (normed, roped) and V rows
  const int64_t rowel = (int64_t)kNKV * kHD;
  if (split == nsplit - 1 && threadIdx.x < kHD) {
    const int64_t off = (a.slot0 + pos) * rowel + h * kHD + threadIdx.x;
    kc[off] = ks[threadIdx.x];
    vc[off] = qkv[3072 + h * kHD + threadIdx.x];
  }
  __syncthreads();

  // 3) one chunk of 32 keys per warp
  const int64_t t0 = (int64_t)(split * kAttSplitChunks + warp) * kAttChunk;
  if (t0 < T) {
    const int64_t t = t0 + lane;
    const bool valid = t < T;
    float s[2] = {-__int_as_float(0x7f800000), -__int_as_float(0x7f800000)};
    if (valid) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + (a.slot0 + t) * rowel + h * kHD);
      const uint4* q0 = reinterpret_cast<const uint4*>(qs[0]);
      const uint4* q1 = reinterpret_cast<const uint4*>(qs[1]);
      float a0 = 0.0f, a1 = 0.0f;
#pragma unroll 4
      for (int v = 0; v < kHD / 8; ++v) {
        const uint4 kv = kr[v];
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
      s[0] = __fmul_rn(a0, kAttnScale);
      s[1] = __fmul_rn(a1, kAttnScale);
    }
    const int nvalid = (int)((T - t0) < kAttChunk ? (T - t0) : kAttChunk);
    float m[2], p[2], l[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      m[hh] = warp_max(s[hh]);
      p[hh] = valid ? q3_expf(__fsub_rn(s[hh], m[hh])) : 0.0f;
      l[hh] = warp_sum(p[hh]);
    }
    float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t* vbase = vc + (a.slot0 + t0) * rowel + h * kHD + 4 * lane;
    for (int tt = 0; tt < nvalid; ++tt) {
      const float p0 = __shfl_sync(0xffffffffu, p[0], tt);
      const float p1 = __shfl_sync(0xffffffffu, p[1], tt);
      const uint2 vv = *reinterpret_cast<const uint2*>(vbase + (int64_t)tt * rowel);
      const float v0 = h2f((uint16_t)(vv.x & 0xffffu)), v1 = h2f((uint16_t)(vv.x >> 16));
      const float v2 = h2f((uint16_t)(vv.y & 0xffffu)), v3 = h2f((uint16_t)(vv.y >> 16));
      o0[0] = __fmaf_rn(p0, v0, o0[0]);
      o0[1] = __fmaf_rn(p0, v1, o0[1]);
      o0[2] = __fmaf_rn(p0, v2, o0[2]);
      o0[3] = __fmaf_rn(p0, v3, o0[3]);
      o1[0] = __fmaf_rn(p1, v0, o1[0]);
      o1[1] = __fmaf_rn(p1, v1, o1[1]);
      o1[2] = __fmaf_rn(p1, v2, o1[2]);
      o1[3] = __fmaf_rn(p1, v3, o1[3]);
    }
    if (lane == 0) {
      cp[warp][0].m = m[0];
      cp[warp][0].l = l[0];
      cp[warp][1].m = m[1];
      cp[warp][1].l = l[1];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      cp[warp][0].o[4 * lane + j] = o0[j];
      cp[warp][1].o[4 * lane + j] = o1[j];
    }
  }
  __syncthreads();

  // 4) merge this split's chunks left to right (warp hh merges q head 2h+hh)
  const int64_t keys_here = T - (int64_t)split * kAttSplit;
  const int nchunk_here = keys_here >= kAttSplit ? kAttSplitChunks
                                                 : (int)((keys_here + kAttChunk - 1) / kAttChunk);
  AttnPartial* gpart = a.part + (((int64_t)b * kNKV + h) * a.max_splits) * 2;
  if (warp < 2) {
    const int hh = warp;
    float m = cp[0][hh].m, l = cp[0][hh].l, o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = cp[0][hh].o[4 * lane + j];
    for (int c = 1; c < nchunk_here; ++c) {
      float ob[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) ob[j] = cp[c][hh].o[4 * lane + j];
      att_merge(m, l, o, cp[c][hh].m, cp[c][hh].l, ob);
    }
    if (nsplit == 1) {
      uint16_t* out = a.out + (int64_t)b * a.out_stride + (2 * h + hh) * kHD;
#pragma unroll
      for (int j = 0; j < 4; ++j) out[4 * lane + j] = f2h(__fdiv_rn(o[j], l));
    } else {
      AttnPartial* gp = gpart + split * 2 + hh;
      if (lane == 0) {
        gp->m = m;
        gp->l = l;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) gp->o[4 * lane + j] = o[j];
    }
  }
  if (nsplit == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int* ctr = a.counters + (int64_t)b * kNKV + h;
    const unsigned prev = atomicAdd(ctr, 1u);
    is_last = (prev == (unsigned)(nsplit - 1));
    if (is_last) *ctr = 0u;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // 5) last CTA of this (sequence, kv head): merge the splits left to right
  if (warp < 2) {
    const int hh = warp;
    const volatile AttnPartial* gp = gpart + hh;
    float m = gp->m, l = gp->l, o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = gp->o[4 * lane + j];
    for (int sp = 1; sp < nsplit; ++sp) {
      const volatile AttnPartial* q = gpart + sp * 2 + hh;
      float ob[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) ob[j] = q->o[4 * lane + j];
      att_merge(m, l, o, q->m, q->l, ob);
    }
    uint16_t* out = a.out + (int64_t)b * a.out_stride + (2 * h + hh) * kHD;
#pragma unroll
    for (int j = 0; j < 4; ++j) out[4 * lane + j] = f2h(__fdiv_rn(o[j], l));
  }
}

}  // namespace q3
