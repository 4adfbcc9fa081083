// q3_persist.cuh -- the whole decode loop of one sequence as ONE persistent,
// cooperative kernel (one CTA per SM).
//
// Per step (model/qwen3_full.mlir:1431-1526) and per layer (:751-864) the
// phases are QKV (RMSNorm + Q|K|V), ATTN (QK-norm + RoPE + KV write +
// attention), O (+ residual), GU (RMSNorm + gate|up + SwiGLU), DOWN
// (+ residual); generating steps end with VOCAB (final RMSNorm + vocab GEMV +
// argmax).  Every phase needs all outputs of the one before, so consumers
// meet at a grid barrier between phases (a monotonic arrival counter in
// global memory; every wait is bounded and reports kErrTimeoutGrid).
//
// Weights never depend on activations, so the producer warp of each CTA
// walks the same schedule ahead of its consumers and streams every weight
// tile it will need into a byte ring in shared memory (1-D bulk copies, TMA
// engine).  While consumers wait at a barrier, the next phases' weights are
// already landing: HBM streaming overlaps the synchronisation.  The ring is
// byte-granular (tiles of 8.5 to 25.5 KB share it) with 32 mbarrier slots.
//
// Each phase reuses the per-tile arithmetic of the standalone kernels, so the
// results are bit-identical to them and to the CPU oracle.
#pragma once

#include "q3_attn.cuh"
#include "q3_common.cuh"
#include "q3_gemv.cuh"

namespace q3 {

constexpr int kRingSlots = 32;
constexpr uint32_t kRingBytes = 192 * 1024;
constexpr size_t kPersistSmem = kRingBytes + 2 * kRingSlots * sizeof(uint64_t) + kRingSlots * 8;

enum PPhase : int { PH_QKV = 0, PH_ATTN = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_VOCAB = 5 };

struct PersistArgs {
  // weights, reference layout
  const uint16_t* token_embd;
  const uint16_t* output_norm;
  const uint16_t* output_T;
  const uint16_t* attn_norm;
  const uint16_t* ffn_norm;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const uint8_t* wq;
  const uint8_t* wk;
  const uint8_t* wv;
  const uint8_t* wo;
  const uint8_t* wgu;
  const uint8_t* wd;
  // decoder state
  uint16_t* kc;
  uint16_t* vc;
  const float* rope_cos;
  const float* rope_sin;
  int64_t S;
  uint16_t* x;
  uint16_t* qkv;
  uint16_t* attn;
  uint16_t* h1;
  uint16_t* act;
  uint16_t* logits;       // optional
  int64_t* tokens;        // [S + 1]
  SeqState* seq;
  ArgmaxPartial* am_part; // [gridDim.x]
  unsigned int* am_counter;
  AttnPartial* att_part;  // [8][max_chunks][2]
  unsigned int* att_counters;
  int max_chunks;
  unsigned int* grid_ctr; // zero at launch
  int* err;
  int n_steps;            // decode steps in this launch
  int vocab_from;         // steps s >= vocab_from end with the vocab head
  // Optional phase trace of step `trace_step`: per (CTA, phase) four global-timer
  // stamps -- barrier arrival, barrier release, inputs ready, work done.
  long long* trace;
  int trace_step;
};

constexpr int kTracePhases = kLayers * 5 + 1;

__device__ __forceinline__ void trace_mark(const PersistArgs& a, int s, int p, int k) {
  if (a.trace != nullptr && s == a.trace_step && threadIdx.x == 0) {
    long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.trace[((int64_t)blockIdx.x * kTracePhases + p) * 4 + k] = t;
  }
}

__host__ __device__ constexpr int phase_tiles(int ph) {
  return ph == PH_QKV ? 512 : ph == PH_O ? 128 : ph == PH_GU ? 384 : ph == PH_DOWN ? 128
       : ph == PH_VOCAB ? kVocab / kTileRows : 0;
}
__host__ __device__ constexpr uint32_t phase_tile_bytes(int ph) {
  return ph == PH_QKV ? 8 * 1088u : ph == PH_O ? 8 * 2176u : ph == PH_GU ? 16 * 1088u
       : ph == PH_DOWN ? 8 * 3264u : ph == PH_VOCAB ? 8 * 2048u : 0u;
}

// Position of a tile in the byte ring: tiles are placed back to back and a
// tile that would straddle the end starts again at offset 0.
struct RingCursor {
  uint64_t alloc = 0;  // bytes handed out so far, wrap padding included
  uint32_t idx = 0;    // tiles handed out so far
  __device__ __forceinline__ uint32_t place(uint32_t sz) {
    uint32_t off = (uint32_t)(alloc % kRingBytes);
    if (off + sz > kRingBytes) {
      alloc += kRingBytes - off;
      off = 0;
    }
    alloc += sz;
    ++idx;
    return off;
  }
};

__device__ __forceinline__ void issue_tile(const PersistArgs& a, int ph, int l, int t, uint8_t* dst,
                                           uint64_t* bar, uint64_t pol) {
  const uint32_t sz = phase_tile_bytes(ph);
  mbar_expect_tx(bar, sz);
  switch (ph) {
    case PH_QKV: {
      const int r0 = t * kTileRows;  // rows 0-2047 q, 2048-3071 k, 3072-4095 v
      const uint8_t* src = r0 < 2048 ? a.wq + l * kBplQ + (int64_t)r0 * 1088
                         : r0 < 3072 ? a.wk + l * kBplKV + (int64_t)(r0 - 2048) * 1088
                                     : a.wv + l * kBplKV + (int64_t)(r0 - 3072) * 1088;
      bulk_g2s(dst, src, sz, bar, pol);
      break;
    }
    case PH_O:
      bulk_g2s(dst, a.wo + l * kBplO + (int64_t)t * sz, sz, bar, pol);
      break;
    case PH_GU: {
      const uint8_t* g = a.wgu + l * kBplGU + (int64_t)t * 8 * 1088;
      bulk_g2s(dst, g, 8 * 1088, bar, pol);
      bulk_g2s(dst + 8 * 1088, g + (int64_t)3072 * 1088, 8 * 1088, bar, pol);
      break;
    }
    case PH_DOWN:
      bulk_g2s(dst, a.wd + l * kBplD + (int64_t)t * sz, sz, bar, pol);
      break;
    case PH_VOCAB:
      bulk_g2s(dst, reinterpret_cast<const uint8_t*>(a.output_T) + (int64_t)t * sz, sz, bar, pol);
      break;
  }
}

// Grid barrier over the consumer warps of all CTAs; `target` = CTAs x
// barriers so far.  Bounded: gives up (and records kErrTimeoutGrid) after
// kSpinCycles, or as soon as any CTA has recorded an error.
__device__ __forceinline__ bool grid_barrier(unsigned int* ctr, unsigned target, int* err,
                                             int* ok_s) {
  consumer_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    int ok = 1;
    const long long t0 = clock64();
    for (;;) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if (*(volatile int*)err != 0) {
        ok = 0;
        break;
      }
      if (clock64() - t0 > kSpinCycles) {
        atomicCAS(err, 0, kErrTimeoutGrid);
        ok = 0;
        break;
      }
    }
    *ok_s = ok;
  }
  consumer_sync();
  return *ok_s != 0;
}

// Input slices in registers from global memory written by other CTAs
// (L2 loads; the L1 is not coherent across CTAs).
template <int G>
__device__ __forceinline__ void load_x_blocks_cg(const uint16_t* x, int lane, uint32_t (&xr)[G][16]) {
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint4* p = reinterpret_cast<const uint4*>(x + 32 * (lane + 32 * g));
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 t = __ldcg(p + v);
      xr[g][4 * v + 0] = t.x;
      xr[g][4 * v + 1] = t.y;
      xr[g][4 * v + 2] = t.z;
      xr[g][4 * v + 3] = t.w;
    }
  }
}

// RMSNorm into shared memory (as cta_rmsnorm_to_smem, L2 loads of x).
__device__ __forceinline__ void cta_rmsnorm_cg(const uint16_t* x, const uint16_t* g, uint16_t* xs,
                                               float* rs) {
  const int tid = threadIdx.x;
  if (tid < kDim / 8) reinterpret_cast<uint4*>(xs)[tid] = __ldcg(reinterpret_cast<const uint4*>(x) + tid);
  consumer_sync();
  if (tid < 32) {
    float ss = 0.0f;
    for (int k = tid; k < kDim; k += 32) {
      const float v = h2f(xs[k]);
      ss = __fmaf_rn(v, v, ss);
    }
    ss = warp_sum(ss);
    if (tid == 0) *rs = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kDim), kEps));
  }
  consumer_sync();
  const float r = *rs;
  for (int k = tid; k < kDim; k += 256) xs[k] = rms_apply(xs[k], g[k], r);
  consumer_sync();
}

__global__ void __launch_bounds__(kGemvThreads, 1) k_decode_persistent(const __grid_constant__ PersistArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
  uint64_t* empty = full + kRingSlots;
  uint64_t* ends = empty + kRingSlots;  // producer-private: ring position after each slot's tile
  __shared__ __align__(16) uint16_t xs[kDim];
  __shared__ __align__(16) AttnSmem asm_;
  __shared__ ArgmaxPartial warp_best[kGemvConsumerWarps];
  __shared__ float rs;
  __shared__ int ok_s, quit_s, last_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRingSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvConsumerWarps);
    }
    fence_mbar_init();
    quit_s = 0;
  }
  __syncthreads();

  if (warp == kGemvConsumerWarps) {
    // ============================ producer ============================
    if (lane != 0) return;
    const uint64_t pol = l2_policy_evict_first();
    RingCursor cur;
    uint32_t head = 0;      // oldest tile not yet seen consumed
    uint64_t freed = 0;     // ring bytes released by consumed tiles
    bool stop = false;
    for (int s = 0; s < a.n_steps && !stop; ++s) {
      const int nph = kLayers * 5 + (s >= a.vocab_from ? 1 : 0);
      for (int p = 0; p < nph && !stop; ++p) {
        const int ph = p < kLayers * 5 ? p % 5 : PH_VOCAB;
        const int l = p < kLayers * 5 ? p / 5 : 0;
        const int nt = phase_tiles(ph);
        const uint32_t sz = phase_tile_bytes(ph);
        for (int t = cta; t < nt && !stop; t += G) {
          // placement of this tile, then wait until its bytes and slot are free
          uint64_t al = cur.alloc;
          uint32_t off = (uint32_t)(al % kRingBytes);
          if (off + sz > kRingBytes) al += kRingBytes - off;
          const uint64_t end = al + sz;
          while (end - freed > kRingBytes || cur.idx - head >= (uint32_t)kRingSlots) {
            const int hs = head % kRingSlots;
            const uint32_t par = (head / kRingSlots) & 1;
            const long long t0 = clock64();
            while (!mbar_try_wait(&empty[hs], par)) {
              if (*(volatile int*)&quit_s) { stop = true; break; }
              if (clock64() - t0 > kSpinCycles) {
                atomicCAS(a.err, 0, kErrTimeoutEmpty);
                stop = true;
                break;
              }
            }
            if (stop) break;
            freed = ends[hs];
            ++head;
          }
          if (stop) break;
          const uint32_t o = cur.place(sz);
          const int slot = (cur.idx - 1) % kRingSlots;
          ends[slot] = cur.alloc;
          issue_tile(a, ph, l, t, ring + o, &full[slot], pol);
        }
      }
    }
    // drain: every issued copy must land before the CTA may exit
    for (uint32_t i = head; i < cur.idx; ++i)
      mbar_wait(&full[i % kRingSlots], (i / kRingSlots) & 1, nullptr, 0);
    return;
  }

  // ============================ consumers ============================
  RingCursor cur;
  unsigned nbar = 0;
  bool first = true;
  int64_t pos = __ldcg(reinterpret_cast<const long long*>(&a.seq->pos));
  bool quit = false;

  auto next_tile = [&](uint32_t sz, uint32_t& base, int& slot) -> bool {
    const uint32_t o = cur.place(sz);
    slot = (cur.idx - 1) % kRingSlots;
    if (!mbar_wait(&full[slot], ((cur.idx - 1) / kRingSlots) & 1, a.err, kErrTimeoutFull))
      return false;
    base = smem_u32(ring + o);
    return true;
  };
  auto release = [&](int slot) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  };

  for (int s = 0; s < a.n_steps && !quit; ++s) {
    const bool vocab = s >= a.vocab_from;
    const int nph = kLayers * 5 + (vocab ? 1 : 0);
    for (int p = 0; p < nph && !quit; ++p) {
      const int ph = p < kLayers * 5 ? p % 5 : PH_VOCAB;
      const int l = p < kLayers * 5 ? p / 5 : 0;
      trace_mark(a, s, p, 0);
      if (!first) {
        ++nbar;
        if (!grid_barrier(a.grid_ctr, nbar * (unsigned)G, a.err, &ok_s)) {
          quit = true;
          break;
        }
      }
      first = false;
      trace_mark(a, s, p, 1);
      if (p == 0 && __ldcg(&a.seq->stop) != 0) {  // the end rule fired in an earlier step
        quit = true;
        break;
      }
      if (p == 0 && (pos < 0 || pos >= a.S)) {
        if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrBadPos);
        quit = true;
        break;
      }
      const int nt = phase_tiles(ph);
      const uint32_t sz = phase_tile_bytes(ph);
      if (ph == PH_QKV) {
        const uint16_t* xin = a.x;
        if (l == 0) {
          int64_t tok = __ldcg(reinterpret_cast<const long long*>(a.tokens) + pos);
          if (tok < 0 || tok >= kVocab) {
            if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrBadToken);
            tok = 0;
          }
          xin = a.token_embd + tok * (int64_t)kDim;
          if (cta == 0 && threadIdx.x < kDim / 8)
            reinterpret_cast<uint4*>(a.x)[threadIdx.x] = reinterpret_cast<const uint4*>(xin)[threadIdx.x];
        }
        cta_rmsnorm_cg(xin, a.attn_norm + l * kDim, xs, &rs);
        uint32_t xr[1][16];
        load_x_blocks<1>(xs, 32, lane, xr);
        trace_mark(a, s, p, 2);
        for (int t = cta; t < nt; t += G) {
          uint32_t base;
          int slot;
          if (!next_tile(sz, base, slot)) { quit = true; break; }
          const float d = q8_row_dot<1, kOrderMlir>(base + 1088u * warp, 32, lane, xr);
          if (lane == 0) a.qkv[t * kTileRows + warp] = f2h(d);
          release(slot);
        }
      } else if (ph == PH_ATTN) {
        if (pos < 0 || pos >= a.S || attn_nchunks(pos) > a.max_chunks) {
          if (threadIdx.x == 0) atomicCAS(a.err, 0, kErrBadPos);
          quit = true;
          break;
        }
        AttnCtx c;
        c.qkv = a.qkv;
        c.q_norm = a.q_norm + l * kHD;
        c.k_norm = a.k_norm + l * kHD;
        c.ct = a.rope_cos + pos * 64;
        c.sn = a.rope_sin + pos * 64;
        c.kc = a.kc;
        c.vc = a.vc;
        c.slot0 = (int64_t)l * a.S;
        c.pos = pos;
        c.out = a.attn;
        c.part = a.att_part;
        c.counters = a.att_counters;
        c.max_chunks = a.max_chunks;
        c.trace = nullptr;
        const int ntask = kNKV * attn_ngroups(pos);
        trace_mark(a, s, p, 2);
        for (int j = cta; j < ntask; j += G) attn_group<false>(c, j % kNKV, j / kNKV, asm_);
      } else if (ph == PH_O) {
        uint32_t xr[2][16];
        load_x_blocks_cg<2>(a.attn, lane, xr);
        trace_mark(a, s, p, 2);
        for (int t = cta; t < nt; t += G) {
          uint32_t base;
          int slot;
          if (!next_tile(sz, base, slot)) { quit = true; break; }
          const float d = q8_row_dot<2, kOrderMlir>(base + 2176u * warp, 64, lane, xr);
          const int row = t * kTileRows + warp;
          if (lane == 0) a.h1[row] = f2h(__fadd_rn(h2f((uint16_t)__ldcg(reinterpret_cast<const unsigned short*>(a.x) + row)), h2f(f2h(d))));
          release(slot);
        }
      } else if (ph == PH_GU) {
        cta_rmsnorm_cg(a.h1, a.ffn_norm + l * kDim, xs, &rs);
        uint32_t xr[1][16];
        load_x_blocks<1>(xs, 32, lane, xr);
        trace_mark(a, s, p, 2);
        for (int t = cta; t < nt; t += G) {
          uint32_t base;
          int slot;
          if (!next_tile(sz, base, slot)) { quit = true; break; }
          const float g = q8_row_dot<1, kOrderMlir>(base + 1088u * warp, 32, lane, xr);
          const float u = q8_row_dot<1, kOrderMlir>(base + 1088u * (kTileRows + warp), 32, lane, xr);
          if (lane == 0) a.act[t * kTileRows + warp] = swiglu_h(f2h(g), f2h(u));
          release(slot);
        }
      } else if (ph == PH_DOWN) {
        uint32_t xr[3][16];
        load_x_blocks_cg<3>(a.act, lane, xr);
        trace_mark(a, s, p, 2);
        for (int t = cta; t < nt; t += G) {
          uint32_t base;
          int slot;
          if (!next_tile(sz, base, slot)) { quit = true; break; }
          const float d = q8_row_dot<3, kOrderMlir>(base + 3264u * warp, 96, lane, xr);
          const int row = t * kTileRows + warp;
          if (lane == 0) a.x[row] = f2h(__fadd_rn(h2f((uint16_t)__ldcg(reinterpret_cast<const unsigned short*>(a.h1) + row)), h2f(f2h(d))));
          release(slot);
        }
      } else {  // PH_VOCAB
        cta_rmsnorm_cg(a.x, a.output_norm, xs, &rs);
        uint16_t xh[kVocabK / 32];
#pragma unroll
        for (int i = 0; i < kVocabK / 32; ++i) xh[i] = xs[lane + 32 * i];
        trace_mark(a, s, p, 2);
        float best_v = -__int_as_float(0x7f800000);
        int64_t best_i = -1;
        for (int t = cta; t < nt; t += G) {
          uint32_t base;
          int slot;
          if (!next_tile(sz, base, slot)) { quit = true; break; }
          const uint32_t row = base + 2048u * warp;
          float acc = 0.0f;
#pragma unroll
          for (int k = 0; k < kVocabK / 32; ++k) acc = fma_h(lds16(row + 2u * (lane + 32 * k)), xh[k], acc);
          acc = warp_sum(acc);
          release(slot);
          const uint16_t lh = f2h(acc);
          const int64_t n = (int64_t)t * kTileRows + warp;
          if (lane == 0 && a.logits != nullptr) a.logits[n] = lh;
          const float lv = h2f(lh);
          if (am_better(lv, n, best_v, best_i)) {
            best_v = lv;
            best_i = n;
          }
        }
        if (quit) break;
        if (lane == 0) {
          warp_best[warp].v = best_v;
          warp_best[warp].i = best_i;
        }
        consumer_sync();
        if (threadIdx.x == 0) {
          float bv = -__int_as_float(0x7f800000);
          int64_t bi = -1;
          for (int w = 0; w < kGemvConsumerWarps; ++w)
            if (am_better(warp_best[w].v, warp_best[w].i, bv, bi)) {
              bv = warp_best[w].v;
              bi = warp_best[w].i;
            }
          a.am_part[cta].v = bv;
          a.am_part[cta].i = bi;
          __threadfence();
          const unsigned prev = atomicAdd(a.am_counter, 1u);
          last_s = (prev == (unsigned)G - 1);
          if (last_s) {
            __threadfence();
            // the last CTA: reduce the partials (a total order: any order works)
            for (int c = 0; c < G; ++c) {
              const float v = __ldcg(&a.am_part[c].v);
              const int64_t ii = __ldcg(reinterpret_cast<const long long*>(&a.am_part[c].i));
              if (am_better(v, ii, bv, bi)) {
                bv = v;
                bi = ii;
              }
            }
            SeqState* st = a.seq;
            a.tokens[pos + 1] = bi;
            if (pos >= st->n_prompt) {
              st->n_gen += 1;
              if (st->n_gen >= st->max_gen || ((st->n_gen % 4) == 0 && bi == st->eos)) st->stop = 1;
            }
            st->pos = pos + 1;
            *a.am_counter = 0u;
          }
        }
        consumer_sync();
      }
      trace_mark(a, s, p, 3);
      if (quit) break;
    }
    if (quit) break;
    pos += 1;
  }
  if (threadIdx.x == 0) quit_s = 1;  // releases a producer still waiting for ring space
  if (!quit && cta == 0 && threadIdx.x == 0) a.seq->pos = pos;
}

}  // namespace q3
