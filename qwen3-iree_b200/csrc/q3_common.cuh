// q3_common.cuh -- shared constants and sm_100a device helpers for the
// Qwen3-0.6B Q8_0 decode kernels.
//
// Numerics contract: the library is built with --fmad=false, so no multiply
// and add is ever fused behind our back; every fused multiply-add below is an
// explicit __fmaf_rn or fma.rn.f32.f16.  f16 rounding is always RNE.  With
// that, each kernel reproduces a documented summation order bit for bit.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace q3 {

// Model constants (model/qwen3_full.mlir:29-64).
constexpr int kLayers = 28;
constexpr int kDim = 1024;
constexpr int kNQ = 16;
constexpr int kNKV = 8;
constexpr int kHD = 128;
constexpr int kFFN = 3072;
constexpr int kVocab = 151936;
constexpr int kQBlk = 32;
constexpr int kQBytes = 34;
// Bytes per layer of each stacked Q8_0 weight (tools/create_q8_irpa.py:176-224).
constexpr int64_t kBplQ = 2228224, kBplKV = 1114112, kBplO = 2228224, kBplGU = 6684672,
                  kBplD = 3342336;
constexpr float kEps = 9.99999997e-7f;                 // f32 of 1e-6
constexpr float kAttnScale = 0.0883883476483184405f;   // rsqrt(128), correctly rounded
constexpr int kAttChunk = 32;                          // keys per warp chunk
constexpr int kAttSplitChunks = 8;                     // chunks per split (one CTA)
constexpr int kAttSplit = kAttChunk * kAttSplitChunks; // 256 keys per split

// Device error word values (the host maps them to Q3_ERR_DEVICE_*).
enum : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,     // a consumer gave up waiting for a TMA stage
  kErrTimeoutEmpty = 2,    // the producer gave up waiting for a free stage
  kErrTimeoutGrid = 3,     // a grid barrier / flag wait gave up
  kErrBadToken = 4,        // token id outside the vocabulary
  kErrBadPos = 5,          // position outside the KV cache
};

// Spin budget for every wait in these kernels, in SM clock cycles (~1 s).
constexpr long long kSpinCycles = 2000000000LL;

// ---------------------------------------------------------------------------
// f16 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }

// acc + a*b with a, b f16 and one rounding to f32 (exact product).
__device__ __forceinline__ float fma_h(uint16_t a, uint16_t b, float acc) {
  asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(a), "h"(b));
  return acc;
}

// Two chained fma_h over packed half2 operands: lo*lo first, then hi*hi.
__device__ __forceinline__ float fma_h2(uint32_t a2, uint32_t b2, float acc) {
  asm("{\n\t.reg .f16 a0, a1, b0, b1;\n\t"
      "mov.b32 {a0, a1}, %1;\n\t"
      "mov.b32 {b0, b1}, %2;\n\t"
      "fma.rn.f32.f16 %0, a0, b0, %0;\n\t"
      "fma.rn.f32.f16 %0, a1, b1, %0;\n\t}"
      : "+f"(acc)
      : "r"(a2), "r"(b2));
  return acc;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// exp(x) by Cody-Waite reduction and a degree-7 Taylor polynomial; the same
// operation sequence as the CPU oracle, so both produce identical bits.
__device__ __forceinline__ float q3_expf(float x) {
  if (x != x) return x;
  if (x > 89.0f) return __int_as_float(0x7f800000);
  if (x < -104.0f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.428606820309417e-6f, r);
  float p = 1.984126984126984e-4f;
  p = __fmaf_rn(p, r, 1.388888888888889e-3f);
  p = __fmaf_rn(p, r, 8.333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.166666666666667e-2f);
  p = __fmaf_rn(p, r, 1.666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int k = (int)n;
  if (k > 127) {
    p = __fmul_rn(p, 2.0f);
    k -= 1;
  }
  if (k < -126) {
    p = __fmul_rn(p, __int_as_float((k + 64 + 127) << 23));
    return __fmul_rn(p, __int_as_float((-64 + 127) << 23));
  }
  return __fmul_rn(p, __int_as_float((k + 127) << 23));
}

// The reference kernels' warp butterfly (offsets 16, 8, 4, 2, 1).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// The same maximum (NaN-free inputs) in one redux.sync on order-preserving
// keys: negative floats map to their complement, others get the sign bit set.
// A max is exact, so only the sign of a zero result can differ from
// warp_max, and a zero's sign does not survive the differences it enters.
__device__ __forceinline__ float warp_max_redux(float v) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  const uint32_t m = __reduce_max_sync(0xffffffffu, key);
  return __uint_as_float((m & 0x80000000u) ? (m & 0x7fffffffu) : ~m);
}

// f16 SwiGLU of model/qwen3_full.mlir:829-839, every op rounded to f16.
__device__ __forceinline__ uint16_t swiglu_h(uint16_t gate, uint16_t up) {
  const float g = h2f(gate);
  const float e = h2f(f2h(q3_expf(-g)));
  const float den = h2f(f2h(__fadd_rn(1.0f, e)));
  const float sig = h2f(f2h(__fdiv_rn(1.0f, den)));
  const float silu = h2f(f2h(__fmul_rn(g, sig)));
  return f2h(__fmul_rn(silu, h2f(up)));
}

// ---------------------------------------------------------------------------
// Shared memory, mbarrier and bulk-copy (TMA) helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `code` in
// *err) if the phase did not complete within kSpinCycles, or if another CTA
// already reported an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > kSpinCycles) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
    if (err && *(volatile int*)err != 0) return false;
  }
}

// Bounded wait that records `code` in *err on timeout but, unlike mbar_wait,
// keeps waiting when some other kernel raised *err: a pipeline role that
// stops early must still see its own copies and MMAs complete.
__device__ __forceinline__ bool mbar_wait_own(uint64_t* bar, uint32_t parity, int* err, int code,
                                              long long limit = kSpinCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > limit) {
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

// Optional per-launch timing record (the graph engine's kernel trace), in ns
// of %globaltimer, kept by thread 0 of every CTA: t[0] first CTA start,
// t[1] first release from the wait on the previous kernel, t[2] last
// release, t[3] last CTA end, t[4] last CTA start, t[5] first CTA end.  A
// null pointer records nothing.
constexpr int kTraceVals = 8;
__device__ __forceinline__ unsigned long long gtimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void ktrace_start(unsigned long long* t) {
  if (t != nullptr && threadIdx.x == 0) {
    const unsigned long long n = gtimer_ns();
    atomicMin(t, n);
    atomicMax(t + 4, n);
  }
}
__device__ __forceinline__ void ktrace_release(unsigned long long* t) {
  if (t != nullptr && threadIdx.x == 0) {
    const unsigned long long n = gtimer_ns();
    atomicMin(t + 1, n);
    atomicMax(t + 2, n);
  }
}
__device__ __forceinline__ void ktrace_end(unsigned long long* t, unsigned tid = 0) {
  if (t != nullptr && threadIdx.x == tid) {
    const unsigned long long n = gtimer_ns();
    atomicMax(t + 3, n);
    atomicMin(t + 5, n);
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> this CTA's shared memory, completion on an mbarrier.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Prefetch a global range into L2 (bulk, no shared memory involved).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.b16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Q8_0 block dot products (one lane, one 34-byte block in shared memory)
// ---------------------------------------------------------------------------
// The block starts at shared byte address `a` (2-byte aligned; 4-byte
// aligned exactly when the block index is even).  Nine aligned words cover
// it; realignment is one byte_perm per word.
struct Q8BlockWords {
  uint32_t q[8];      // the 32 int8 values, 4 per word, in order
  uint32_t scale16;   // f16 bits of the scale in the low half
};

__device__ __forceinline__ Q8BlockWords q8_load_block(uint32_t a) {
  const uint32_t base = a & ~3u;
  const bool odd = (a & 2u) != 0;  // qs start 4-byte aligned
  uint32_t w[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) w[i] = lds32(base + 4u * i);
  Q8BlockWords b;
  b.scale16 = odd ? (w[0] >> 16) : (w[0] & 0xffffu);
  const uint32_t sel = odd ? 0x7654u : 0x5432u;
#pragma unroll
  for (int i = 0; i < 8; ++i) b.q[i] = __byte_perm(w[i], w[i + 1], sel);
  return b;
}

// Four int8 (one word) -> two half2 words holding them exactly.
__device__ __forceinline__ void q8x4_to_h2(uint32_t qw, uint32_t& h01, uint32_t& h23) {
  const uint32_t u = qw ^ 0x80808080u;               // offset binary: q + 128
  const uint32_t b01 = __byte_perm(u, 0x64646464u, 0x5140u);  // (1024+u0, 1024+u1)
  const uint32_t b23 = __byte_perm(u, 0x64646464u, 0x7362u);
  h01 = hsub2_u32(b01, 0x64806480u);                  // minus 1152 -> q exactly
  h23 = hsub2_u32(b23, 0x64806480u);
}

// Four int8 (one word) -> four exact f32.
__device__ __forceinline__ void q8x4_to_f32(uint32_t qw, float (&f)[4]) {
  const uint32_t u = qw ^ 0x80808080u;
  f[0] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4b000000u, 0x7650u)), 8388736.0f);
  f[1] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4b000000u, 0x7651u)), 8388736.0f);
  f[2] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4b000000u, 0x7652u)), 8388736.0f);
  f[3] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4b000000u, 0x7653u)), 8388736.0f);
}

// Block dot in the GPU-dialect kernels' order (kernels/mlir/dispatch_12_gpu.mlir:
// 100-129): inner = fma chain of q_j*x_j over j, then acc = fma(scale, inner, acc).
// xr: the block's 32 x values as 16 packed half2.
__device__ __forceinline__ float q8_block_dot_mlir(const Q8BlockWords& b, const uint32_t* xr,
                                                   float acc) {
  float inner = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t h01, h23;
    q8x4_to_h2(b.q[i], h01, h23);
    inner = fma_h2(h01, xr[2 * i], inner);
    inner = fma_h2(h23, xr[2 * i + 1], inner);
  }
  return __fmaf_rn(h2f((uint16_t)b.scale16), inner, acc);
}

// Block dot in the CUDA kernels' order (kernels/cuda/dispatch_3.cu:33-43):
// acc = fma(scale*q_j, x_j, acc) per element (scale*q_j is exact in f32).
// xf: the block's 32 x values as f32.
__device__ __forceinline__ float q8_block_dot_cuda(const Q8BlockWords& b, const float* xf,
                                                   float acc) {
  const float s = h2f((uint16_t)b.scale16);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float f[4];
    q8x4_to_f32(b.q[i], f);
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = __fmaf_rn(__fmul_rn(s, f[j]), xf[4 * i + j], acc);
  }
  return acc;
}

// ---------------------------------------------------------------------------
// Thread-block clusters: barrier and distributed shared memory (DSMEM)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `local_addr` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}
__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, uint32_t rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(dsmem_map(local_addr, rank)) : "memory");
  return v;
}
// 16-byte store into CTA `rank`'s shared memory at the address `local_addr`
// has in this CTA (16-byte aligned).  Remote stores are posted: a cluster
// barrier (arrive.release / wait.acquire) makes them visible to the target.
__device__ __forceinline__ void st_dsmem_v4(uint32_t local_addr, uint32_t rank, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dsmem_map(local_addr, rank)),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
// 16-byte asynchronous store into CTA `rank`'s shared memory whose arrival
// completes `bytes` on that CTA's mbarrier (the address `local_bar` has in
// this CTA): the receiver waits on its own barrier, no cluster barrier needed.
__device__ __forceinline__ void st_async_v4(uint32_t local_addr, uint32_t rank, uint4 v,
                                            uint32_t local_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          dsmem_map(local_addr, rank)),
      "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(dsmem_map(local_bar, rank))
      : "memory");
}
__device__ __forceinline__ uint16_t ld_dsmem_u16(uint32_t local_addr, uint32_t rank) {
  uint16_t v;
  asm volatile("ld.shared::cluster.u16 %0, [%1];" : "=h"(v) : "r"(dsmem_map(local_addr, rank)) : "memory");
  return v;
}

}  // namespace q3
