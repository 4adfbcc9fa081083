// q3_attn.cuh -- GQA decode attention for sm_100a.
//
// Replaces, for one layer and one or more independent sequences:
//   QK-RMSNorm (model/qwen3_full.mlir:646-702), RoPE (:324-454), the KV-cache
//   write at slot layer*S + pos (:793-797) and iree_linalg_ext.attention over
//   keys 0..pos (:456-530), with the reference's whole-slice KV copy
//   (:715-720) removed: the kernel attends straight out of the flat cache.
//
// Flash decode over chunks of 32 keys.  A group (one CTA, 8 warps) owns 8
// consecutive chunks of one kv head h; each warp turns one chunk into a
// partial (m, l, o[128]) for both q heads 2h and 2h+1, so every K/V row is
// read once (lane = key for q.k, lane = 4 head dims for p.v; a chunk's loads
// are issued before everything else the CTA does).  The CTA folds its chunk
// partials left to right in shared memory; with one group (pos < 256) that is
// the result, otherwise it publishes the group partial and the CTA that
// finishes last for head h (an arrival counter, no spin-waits) folds the
// group partials left to right, loading eight at a time.  The CPU oracle
// (q3o_attention) states the same two-level order, so any assignment of
// groups to CTAs gives the same bits.
#pragma once

#include "q3_common.cuh"
#include "q3_gemv.cuh"

namespace q3 {

struct AttnPartial {  // 528 bytes: o first so the float4 accesses stay 16-byte aligned
  float o[kHD];
  float m, l;
  float pad[2];
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
  AttnPartial* part;        // [B][8][max_chunks][2] chunk partials
  unsigned int* counters;   // [B][8], zero between launches
  int max_chunks;           // >= ceil(S / 32)
  int* err;
  unsigned long long* trace;  // optional launch timing record (4 values)
};

// Everything one group needs about one (sequence, layer).
struct AttnCtx {
  const uint16_t* qkv;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const float* ct;  // RoPE cos row at pos
  const float* sn;  // RoPE sin row at pos
  uint16_t* kc;
  uint16_t* vc;
  int64_t slot0;
  int64_t pos;
  uint16_t* out;
  AttnPartial* part;      // [8][max_chunks][2]
  unsigned int* counters; // [8]
  int max_chunks;
  unsigned long long* trace;  // optional launch timing record
};

struct AttnSmem {
  AttnPartial part[kAttSplitChunks][2];  // this CTA's chunk partials when it holds every chunk
  uint16_t qs[2][kHD];
  uint16_t ks[kHD];
  float2 pw[kAttSplitChunks][kAttChunk];  // each warp's softmax weights, both q heads
  int last;
};

__device__ __forceinline__ int attn_nchunks(int64_t pos) { return (int)((pos + kAttChunk) / kAttChunk); }
__device__ __forceinline__ int attn_ngroups(int64_t pos) {
  return (attn_nchunks(pos) + kAttSplitChunks - 1) / kAttSplitChunks;
}

// Per-head RMSNorm (f16 out) then NeoX RoPE (f16 out) for one 128-wide head.
// Lane l produces outputs l, l+32, l+64, l+96.
__device__ __forceinline__ void head_norm_rope(const uint16_t* x, const uint16_t* g, float c0,
                                               float s0, float c1, float s1, int lane,
                                               uint16_t* dst) {
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = h2f(__ldcg(reinterpret_cast<const unsigned short*>(x) + lane + 32 * i));
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

// The same with this lane's gamma values g[lane + 32 i] already in registers.
__device__ __forceinline__ void head_norm_rope_g(const uint16_t* x, const uint16_t (&gv)[4],
                                                 float c0, float s0, float c1, float s1, int lane,
                                                 uint16_t* dst) {
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = h2f(__ldcg(reinterpret_cast<const unsigned short*>(x) + lane + 32 * i));
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

// The same with the head's values v[i] = x[lane + 32 i] already loaded.
__device__ __forceinline__ void norm_rope_vals(const float (&v)[4], const uint16_t (&gv)[4], float c0,
                                               float s0, float c1, float s1, int lane,
                                               uint16_t* dst) {
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

// Fold the first n partials of a group held in shared memory, left to right.
__device__ __forceinline__ void fold_smem(const AttnSmem& sm, int n, int hh, int lane, float& m,
                                          float& l, float (&o)[4]) {
  m = sm.part[0][hh].m;
  l = sm.part[0][hh].l;
  {
    const float4 t4 = *reinterpret_cast<const float4*>(&sm.part[0][hh].o[4 * lane]);
    o[0] = t4.x, o[1] = t4.y, o[2] = t4.z, o[3] = t4.w;
  }
  for (int k = 1; k < n; ++k) {
    const AttnPartial& q = sm.part[k][hh];
    const float4 t4 = *reinterpret_cast<const float4*>(&q.o[4 * lane]);
    const float ob[4] = {t4.x, t4.y, t4.z, t4.w};
    att_merge(m, l, o, q.m, q.l, ob);
  }
}

// One group (kv head h, chunks 8g .. 8g+7) on the 256 consumer threads of a
// CTA.  Must be called by all of them.  Returns after the head's output is
// written if this CTA was the last of head h, else after its group partial is.
// EARLY: issue the K/V loads before the norms (latency hidden, more live
// registers); otherwise right after them.  Both give the same bits.
template <bool EARLY>
__device__ __forceinline__ void attn_group(const AttnCtx& c, int h, int g, AttnSmem& sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pos = c.pos, T = pos + 1;
  const int nch = attn_nchunks(pos);
  const int ngroups = attn_ngroups(pos);
  const int64_t rowel = (int64_t)kNKV * kHD;
  const int ci = g * kAttSplitChunks + warp;
  const bool have = ci < nch;
  const int64_t t0 = (int64_t)ci * kAttChunk;
  const int64_t t = t0 + lane;
  const bool valid = have && t < T;
  const int nvalid = !have ? 0 : (int)((T - t0) < kAttChunk ? (T - t0) : kAttChunk);

  // 0) this warp's K/V loads go out first (they do not depend on the norms
  //    below): this lane's K row, and 4 dims of every V row of the chunk.  Key
  //    pos is written by this launch and is substituted after step 1.
  uint4 kv[kHD / 8];
  uint2 vv[kAttChunk];
  auto load_chunk = [&]() {
    const uint4* kr = reinterpret_cast<const uint4*>(c.kc + (c.slot0 + (valid ? t : t0)) * rowel + h * kHD);
#pragma unroll
    for (int v = 0; v < kHD / 8; ++v) kv[v] = __ldcg(kr + v);
    const uint16_t* vbase = c.vc + (c.slot0 + t0) * rowel + h * kHD + 4 * lane;
#pragma unroll
    for (int tt = 0; tt < kAttChunk; ++tt)
      vv[tt] = tt < nvalid ? __ldcg(reinterpret_cast<const uint2*>(vbase + (int64_t)tt * rowel))
                           : make_uint2(0u, 0u);
  };
  // key pos of this chunk (if any) is taken from the projection, not the cache
  const int tp = (have && pos < t0 + kAttChunk) ? (int)(pos - t0) : -1;
  // RoPE angles and norm gammas are constants: read them with the K/V loads
  float rc0 = 0.f, rs0 = 0.f, rc1 = 0.f, rs1 = 0.f;
  uint16_t gv[4] = {0, 0, 0, 0};
  if (warp < 3) {
    rc0 = c.ct[lane], rs0 = c.sn[lane], rc1 = c.ct[lane + 32], rs1 = c.sn[lane + 32];
    const uint16_t* g = warp < 2 ? c.q_norm : c.k_norm;
#pragma unroll
    for (int i = 0; i < 4; ++i) gv[i] = g[lane + 32 * i];
  }
  if (EARLY) {
    if (have) load_chunk();
    // cache rows below pos were written by earlier launches: the loads above
    // went out before the wait; q, k, v come from the previous kernel
    pdl_wait();
    ktrace_release(c.trace);
  }
  uint2 nv = make_uint2(0u, 0u);  // the new V row's dims 4 lane .. 4 lane + 3
  if (tp >= 0) nv = __ldcg(reinterpret_cast<const uint2*>(c.qkv + 3072 + h * kHD + 4 * lane));
  // the new V row for the cache write of step 2, fetched now so that its
  // latency overlaps the norms instead of delaying warps 0-3 after them
  const bool writes_row = g == ngroups - 1 && threadIdx.x < kHD;
  unsigned short vrow = 0;
  if (writes_row)
    vrow = __ldcg(reinterpret_cast<const unsigned short*>(c.qkv) + 3072 + h * kHD + threadIdx.x);

  // 1) q heads 2h, 2h+1 and k head h: norm + rope into shared memory
  if (warp < 3) {
    if (warp < 2)
      head_norm_rope_g(c.qkv + (2 * h + warp) * kHD, gv, rc0, rs0, rc1, rs1, lane, sm.qs[warp]);
    else
      head_norm_rope_g(c.qkv + 2048 + h * kHD, gv, rc0, rs0, rc1, rs1, lane, sm.ks);
  }
  consumer_sync();
  // 2) the group holding key pos writes the new K (normed, roped) and V rows,
  //    and the warp holding it takes them from here instead of its stale loads
  if (writes_row) {
    const int64_t off = (c.slot0 + pos) * rowel + h * kHD + threadIdx.x;
    c.kc[off] = sm.ks[threadIdx.x];
    c.vc[off] = vrow;
  }
  if (!EARLY && have) load_chunk();
  if (lane == tp) {
#pragma unroll
    for (int v = 0; v < kHD / 8; ++v) kv[v] = reinterpret_cast<const uint4*>(sm.ks)[v];
  }

  // 3) one chunk of 32 keys per warp -> its partial in shared memory
  if (have) {
    float s[2] = {-__int_as_float(0x7f800000), -__int_as_float(0x7f800000)};
    if (valid) {
      const uint4* q0 = reinterpret_cast<const uint4*>(sm.qs[0]);
      const uint4* q1 = reinterpret_cast<const uint4*>(sm.qs[1]);
      float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
      for (int v = 0; v < kHD / 8; ++v) {
        const uint4 x0 = q0[v], x1 = q1[v];
        a0 = fma_h2(x0.x, kv[v].x, a0);
        a0 = fma_h2(x0.y, kv[v].y, a0);
        a0 = fma_h2(x0.z, kv[v].z, a0);
        a0 = fma_h2(x0.w, kv[v].w, a0);
        a1 = fma_h2(x1.x, kv[v].x, a1);
        a1 = fma_h2(x1.y, kv[v].y, a1);
        a1 = fma_h2(x1.z, kv[v].z, a1);
        a1 = fma_h2(x1.w, kv[v].w, a1);
      }
      s[0] = __fmul_rn(a0, kAttnScale);
      s[1] = __fmul_rn(a1, kAttnScale);
    }
    float m[2], p[2], l[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      m[hh] = warp_max_redux(s[hh]);
      p[hh] = valid ? q3_expf(__fsub_rn(s[hh], m[hh])) : 0.0f;
      l[hh] = warp_sum(p[hh]);
    }
    // p.v, lane = 4 head dims, keys in order.  The weights go through shared
    // memory (one broadcast load per key instead of two shuffles) and the
    // loop has no branch, so its loads issue ahead of the FMA chains; keys
    // past the chunk's end have p = 0 and V = 0 and add an exact +0.
    sm.pw[warp][lane] = make_float2(p[0], p[1]);
    __syncwarp();
    float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int tt = 0; tt < kAttChunk; ++tt) {
      const float2 pp = sm.pw[warp][tt];
      const uint2 vt = tt == tp ? nv : vv[tt];
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
    AttnPartial* gp = sm.part[warp];
    if (lane == 0) {
      gp[0].m = m[0];
      gp[0].l = l[0];
      gp[1].m = m[1];
      gp[1].l = l[1];
    }
    *reinterpret_cast<float4*>(&gp[0].o[4 * lane]) = make_float4(o0[0], o0[1], o0[2], o0[3]);
    *reinterpret_cast<float4*>(&gp[1].o[4 * lane]) = make_float4(o1[0], o1[1], o1[2], o1[3]);
  }
  consumer_sync();

  // 4) fold this group's chunks left to right (warps 0, 1: q heads 2h, 2h+1)
  float m, l, o[4];
  const int hh = warp;
  if (warp < 2) {
    const int ng = nch - g * kAttSplitChunks < kAttSplitChunks ? nch - g * kAttSplitChunks
                                                               : kAttSplitChunks;
    fold_smem(sm, ng, hh, lane, m, l, o);
  }
  if (ngroups > 1) {
    // 5) publish the group partial; the CTA that finishes last for head h
    //    folds the group partials left to right
    AttnPartial* gpart = c.part + ((int64_t)h * c.max_chunks + g) * 2;
    if (warp < 2) {
      if (lane == 0) {
        gpart[hh].m = m;
        gpart[hh].l = l;
      }
      *reinterpret_cast<float4*>(&gpart[hh].o[4 * lane]) = make_float4(o[0], o[1], o[2], o[3]);
    }
    consumer_sync();  // the partial stores precede thread 0's release
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(c.counters + h, 1u);
      sm.last = (prev == (unsigned)(ngroups - 1));
      if (sm.last) c.counters[h] = 0u;
      __threadfence();
    }
    consumer_sync();
    if (!sm.last || warp >= 2) return;
    const AttnPartial* base = c.part + (int64_t)h * c.max_chunks * 2 + hh;
    m = __ldcg(&base->m);
    l = __ldcg(&base->l);
    {
      const float4 t4 = __ldcg(reinterpret_cast<const float4*>(&base->o[4 * lane]));
      o[0] = t4.x, o[1] = t4.y, o[2] = t4.z, o[3] = t4.w;
    }
    for (int k0 = 1; k0 < ngroups; k0 += 8) {  // the loads of eight groups before their merges
      float4 ob4[8];
      float mb[8], lb[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (k0 + u < ngroups) {
          const AttnPartial* q = base + (int64_t)(k0 + u) * 2;
          ob4[u] = __ldcg(reinterpret_cast<const float4*>(&q->o[4 * lane]));
          mb[u] = __ldcg(&q->m);
          lb[u] = __ldcg(&q->l);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (k0 + u < ngroups) {
          const float ob[4] = {ob4[u].x, ob4[u].y, ob4[u].z, ob4[u].w};
          att_merge(m, l, o, mb[u], lb[u], ob);
        }
      }
    }
  }
  if (warp < 2) {
    uint16_t* out = c.out + (2 * h + hh) * kHD + 4 * lane;
    uint2 pk;
    pk.x = (uint32_t)f2h(__fdiv_rn(o[0], l)) | ((uint32_t)f2h(__fdiv_rn(o[1], l)) << 16);
    pk.y = (uint32_t)f2h(__fdiv_rn(o[2], l)) | ((uint32_t)f2h(__fdiv_rn(o[3], l)) << 16);
    *reinterpret_cast<uint2*>(out) = pk;
  }
}

// Standalone launch: grid (8 kv heads, max groups, sequences), 256 threads.
template <bool EARLY>
__global__ void __launch_bounds__(256, EARLY ? 1 : 2) k_attn_decode(const __grid_constant__ AttnArgs a) {
  __shared__ __align__(16) AttnSmem sm;
  const int h = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  ktrace_start(a.trace);
  pdl_launch_dependents();
  // stop and pos change only in a decode step's last kernel: with EARLY they
  // and the K/V loads go before the wait (inside attn_group)
  if (!EARLY) {
    pdl_wait();
    ktrace_release(a.trace);
  }
  if (a.stop != nullptr && a.stop[(int64_t)b * a.stop_stride] != 0) return;
  const int64_t pos = a.pos[(int64_t)b * a.pos_stride];
  if (pos < 0 || pos >= a.S || pos >= a.rope_pos ||
      attn_nchunks(pos) > a.max_chunks) {
    if (threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, kErrBadPos);
    return;
  }
  if (g >= attn_ngroups(pos)) return;
  AttnCtx c;
  c.qkv = a.qkv + (int64_t)b * a.qkv_stride;
  c.q_norm = a.q_norm;
  c.k_norm = a.k_norm;
  c.ct = a.rope_cos + pos * 64;
  c.sn = a.rope_sin + pos * 64;
  c.kc = a.kc + (int64_t)b * a.cache_stride;
  c.vc = a.vc + (int64_t)b * a.cache_stride;
  c.slot0 = a.slot0;
  c.pos = pos;
  c.out = a.out + (int64_t)b * a.out_stride;
  c.part = a.part + (int64_t)b * kNKV * a.max_chunks * 2;
  c.counters = a.counters + (int64_t)b * kNKV;
  c.max_chunks = a.max_chunks;
  c.trace = a.trace;
  attn_group<EARLY>(c, h, g, sm);
  ktrace_end(a.trace);
}

}  // namespace q3
