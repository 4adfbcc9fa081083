// ref_launch.cu -- host launchers for the reference's own CUDA kernels
// (kernels/cuda/dispatch_{3,4,12,18,20,24}.cu, compiled unchanged from the
// reference tree by oracle/Makefile).  TEST INFRASTRUCTURE ONLY: the GPU
// tests run these to pin the CPU oracle against the reference itself.
// Each launcher reproduces the IREE launch of cuda/dispatch_N.mlir: grid
// N/8 x 256 threads, bindings b0/b1/b2 as raw device pointers.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

extern "C" __global__ void decode_dispatch_3_matmul_2048x1x1024_f16(const uint8_t*, const char*,
                                                                    char*, uint32_t, uint32_t);
extern "C" __global__ void decode_dispatch_4_matmul_1024x1x1024_f16(const uint8_t*, const char*,
                                                                    char*, uint32_t, uint32_t,
                                                                    uint32_t);
extern "C" __global__ void decode_dispatch_12_matmul_1024x1x2048_f16(const uint8_t*, const char*,
                                                                     char*, uint32_t, uint32_t);
extern "C" __global__ void decode_dispatch_18_matmul_6144x1x1024_f16(const uint8_t*, const char*,
                                                                     char*, uint32_t, uint32_t);
extern "C" __global__ void decode_dispatch_20_matmul_1024x1x3072_f16(const uint8_t*, const char*,
                                                                     char*, uint32_t, uint32_t);
extern "C" __global__ void decode_dispatch_24_matmul_151936x1x1024_f16(const __half*, const char*,
                                                                       char*, uint32_t);

#define RET return (int)cudaGetLastError()
extern "C" int ref_dispatch_3(const void* w, const void* b1, void* b2, uint32_t c0, uint32_t c1,
                              void* s) {
  decode_dispatch_3_matmul_2048x1x1024_f16<<<256, 256, 0, (cudaStream_t)s>>>(
      (const uint8_t*)w, (const char*)b1, (char*)b2, c0, c1);
  RET;
}
extern "C" int ref_dispatch_4(const void* w, const void* b1, void* b2, uint32_t c0, uint32_t c1,
                              uint32_t c2, void* s) {
  decode_dispatch_4_matmul_1024x1x1024_f16<<<128, 256, 0, (cudaStream_t)s>>>(
      (const uint8_t*)w, (const char*)b1, (char*)b2, c0, c1, c2);
  RET;
}
extern "C" int ref_dispatch_12(const void* w, const void* b1, void* b2, uint32_t c0, uint32_t c1,
                               void* s) {
  decode_dispatch_12_matmul_1024x1x2048_f16<<<128, 256, 0, (cudaStream_t)s>>>(
      (const uint8_t*)w, (const char*)b1, (char*)b2, c0, c1);
  RET;
}
extern "C" int ref_dispatch_18(const void* w, const void* b1, void* b2, uint32_t c0, uint32_t c1,
                               void* s) {
  decode_dispatch_18_matmul_6144x1x1024_f16<<<768, 256, 0, (cudaStream_t)s>>>(
      (const uint8_t*)w, (const char*)b1, (char*)b2, c0, c1);
  RET;
}
extern "C" int ref_dispatch_20(const void* w, const void* b1, void* b2, uint32_t c0, uint32_t c1,
                               void* s) {
  decode_dispatch_20_matmul_1024x1x3072_f16<<<128, 256, 0, (cudaStream_t)s>>>(
      (const uint8_t*)w, (const char*)b1, (char*)b2, c0, c1);
  RET;
}
extern "C" int ref_dispatch_24(const void* w, const void* b1, void* b2, uint32_t c0, void* s) {
  decode_dispatch_24_matmul_151936x1x1024_f16<<<18992, 256, 0, (cudaStream_t)s>>>(
      (const __half*)w, (const char*)b1, (char*)b2, c0);
  RET;
}
