// q3_iree.cuh -- sm_100a replacements of the reference's six substituted IREE
// executables, with the export names, parameter lists and fixed launch
// (grid N/8 x 256 threads) of kernels/cuda/dispatch_{3,4,12,18,20,24}.cu and
// cuda/dispatch_*.mlir count().  One launch per dispatch, as the IREE route
// requires.  Each CTA owns 8 rows: one bulk copy (TMA engine) brings their
// contiguous bytes into shared memory while the warps load their input slice;
// warp w then reduces row 8*blockIdx.x + w in the reference kernels' own
// summation order, so outputs match them bit for bit.
#pragma once

#include "q3_common.cuh"
#include "q3_gemv.cuh"

namespace q3 {

template <int N, int K>
__device__ __forceinline__ void iree_q8_body(const uint8_t* q8_stacked, const char* b1, char* b2,
                                             int64_t layer, int64_t in_off, int64_t out_off,
                                             int64_t bpl) {
  constexpr int nb = K / kQBlk;
  constexpr uint32_t rowbytes = nb * kQBytes;
  constexpr int G = (K + 1023) / 1024;
  __shared__ __align__(128) uint8_t tile[kTileRows * rowbytes];
  __shared__ __align__(8) uint64_t bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kTileRows;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (row0 >= N) return;
  if (threadIdx.x == 0) {
    mbar_expect_tx(&bar, kTileRows * rowbytes);
    bulk_g2s(tile, q8_stacked + layer * bpl + (int64_t)row0 * rowbytes, kTileRows * rowbytes, &bar,
             l2_policy_evict_first());
  }
  uint32_t xr[G][16];
  load_x_blocks<G>(reinterpret_cast<const uint16_t*>(b1 + in_off), nb, lane, xr);
  if (!mbar_wait(&bar, 0u, nullptr, 0)) return;
  const float d = q8_row_dot<G, kOrderCuda>(smem_u32(tile) + rowbytes * warp, nb, lane, xr);
  if (lane == 0) reinterpret_cast<uint16_t*>(b2 + out_off)[row0 + warp] = f2h(d);
}

__device__ __forceinline__ void iree_f16_body(const uint16_t* weight, const char* b1, char* b2,
                                              int64_t out_off) {
  constexpr int N = kVocab, K = 1024;
  constexpr uint32_t rowbytes = K * 2;
  __shared__ __align__(128) uint8_t tile[kTileRows * rowbytes];
  __shared__ __align__(8) uint64_t bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kTileRows;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (row0 >= N) return;
  if (threadIdx.x == 0) {
    mbar_expect_tx(&bar, kTileRows * rowbytes);
    bulk_g2s(tile, reinterpret_cast<const uint8_t*>(weight) + (int64_t)row0 * rowbytes,
             kTileRows * rowbytes, &bar, l2_policy_evict_first());
  }
  const uint16_t* x = reinterpret_cast<const uint16_t*>(b1 + 64);
  uint16_t xh[K / 32];
#pragma unroll
  for (int i = 0; i < K / 32; ++i) xh[i] = x[lane + 32 * i];
  if (!mbar_wait(&bar, 0u, nullptr, 0)) return;
  const uint32_t row = smem_u32(tile) + rowbytes * warp;
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < K / 32; ++i) acc = fma_h(lds16(row + 2u * (lane + 32 * i)), xh[i], acc);
  acc = warp_sum(acc);
  if (lane == 0) reinterpret_cast<uint16_t*>(b2 + out_off)[row0 + warp] = f2h(acc);
}

}  // namespace q3

// Export names and parameters of kernels/cuda/dispatch_*.cu.
extern "C" __global__ void __launch_bounds__(256)
    decode_dispatch_3_matmul_2048x1x1024_f16(const uint8_t* __restrict__ q8_stacked,
                                             const char* __restrict__ b1_raw,
                                             char* __restrict__ b2_raw, uint32_t c0, uint32_t c1) {
  const int64_t layer = (int64_t)((uint64_t)c0 | ((uint64_t)c1 << 32));
  q3::iree_q8_body<2048, 1024>(q8_stacked, b1_raw, b2_raw, layer, 2112, 4160, q3::kBplQ);
}

extern "C" __global__ void __launch_bounds__(256)
    decode_dispatch_4_matmul_1024x1x1024_f16(const uint8_t* __restrict__ q8_stacked,
                                             const char* __restrict__ b1_raw,
                                             char* __restrict__ b2_raw, uint32_t c0, uint32_t c1,
                                             uint32_t c2) {
  const int64_t layer = (int64_t)((uint64_t)c1 | ((uint64_t)c2 << 32));
  q3::iree_q8_body<1024, 1024>(q8_stacked, b1_raw, b2_raw, layer, 2112, (int64_t)(int32_t)c0,
                               q3::kBplKV);
}

extern "C" __global__ void __launch_bounds__(256)
    decode_dispatch_12_matmul_1024x1x2048_f16(const uint8_t* __restrict__ q8_stacked,
                                              const char* __restrict__ b1_raw,
                                              char* __restrict__ b2_raw, uint32_t c0, uint32_t c1) {
  const int64_t layer = (int64_t)((uint64_t)c0 | ((uint64_t)c1 << 32));
  q3::iree_q8_body<1024, 2048>(q8_stacked, b1_raw, b2_raw, layer, 12352, 2048, q3::kBplO);
}

extern "C" __global__ void __launch_bounds__(256)
    decode_dispatch_18_matmul_6144x1x1024_f16(const uint8_t* __restrict__ q8_stacked,
                                              const char* __restrict__ b1_raw,
                                              char* __restrict__ b2_raw, uint32_t c0, uint32_t c1) {
  const int64_t layer = (int64_t)((uint64_t)c0 | ((uint64_t)c1 << 32));
  q3::iree_q8_body<6144, 1024>(q8_stacked, b1_raw, b2_raw, layer, 64, 6144, q3::kBplGU);
}

extern "C" __global__ void __launch_bounds__(256)
    decode_dispatch_20_matmul_1024x1x3072_f16(const uint8_t* __restrict__ q8_stacked,
                                              const char* __restrict__ b1_raw,
                                              char* __restrict__ b2_raw, uint32_t c0, uint32_t c1) {
  const int64_t layer = (int64_t)((uint64_t)c0 | ((uint64_t)c1 << 32));
  q3::iree_q8_body<1024, 3072>(q8_stacked, b1_raw, b2_raw, layer, 18432, 0, q3::kBplD);
}

extern "C" __global__ void __launch_bounds__(256)
    decode_dispatch_24_matmul_151936x1x1024_f16(const __half* __restrict__ weight,
                                                const char* __restrict__ b1_raw,
                                                char* __restrict__ b2_raw, uint32_t c0) {
  q3::iree_f16_body(reinterpret_cast<const uint16_t*>(weight), b1_raw, b2_raw,
                    (int64_t)(int32_t)c0);
}
