// q3_api.cu -- the C ABI of libq3b200.so (include/q3b200.h): launchers for
// the sm_100a kernels, the IREE-ABI dispatch launchers, and the decoder
// object that runs the reference's @run / @decode / @chat_turn semantics as
// CUDA graphs of the fused kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>
#include <thread>
#include <vector>

#include "q3_attn.cuh"
#include "q3_common.cuh"
#include "q3_fused.cuh"
#include "q3_gemv.cuh"
#include "q3_iree.cuh"
#include "q3_persist.cuh"
#include "q3b200.h"

using namespace q3;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local char g_err[512] = "";

static int set_err(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

#define Q3_CUDA(call)                                                                     \
  do {                                                                                    \
    cudaError_t e_ = (call);                                                              \
    if (e_ != cudaSuccess)                                                                \
      return set_err(Q3_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                     __FILE__, __LINE__);                                                 \
  } while (0)

#define Q3_LAUNCHED()                                                                    \
  do {                                                                                   \
    cudaError_t e_ = cudaGetLastError();                                                 \
    if (e_ != cudaSuccess)                                                               \
      return set_err(Q3_ERR_CUDA, "kernel launch failed: %s (%s:%d)",                    \
                     cudaGetErrorString(e_), __FILE__, __LINE__);                        \
  } while (0)

#define Q3_REQUIRE(cond, ...)                              \
  do {                                                     \
    if (!(cond)) return set_err(Q3_ERR_INVALID, __VA_ARGS__); \
  } while (0)

static inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

extern "C" const char* q3_strerror(int s) {
  switch (s) {
    case Q3_OK: return "ok";
    case Q3_ERR_INVALID: return "invalid argument";
    case Q3_ERR_CUDA: return "CUDA runtime error";
    case Q3_ERR_DEVICE: return "kernel reported an error (wait limit, bad token or position)";
    case Q3_ERR_NOMEM: return "out of memory";
    case Q3_ERR_STATE: return "call out of sequence";
    case Q3_ERR_UNSUPPORTED: return "unsupported device or shape";
    default: return "unknown status";
  }
}
extern "C" const char* q3_last_error(void) { return g_err; }
extern "C" int q3_abi_version(void) { return Q3B200_ABI_VERSION; }

// ---------------------------------------------------------------------------
// device plumbing
// ---------------------------------------------------------------------------
extern "C" int q3_device_count(int* n) {
  Q3_REQUIRE(n, "n is null");
  *n = 0;
  cudaError_t e = cudaGetDeviceCount(n);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    *n = 0;
    cudaGetLastError();
    return Q3_OK;
  }
  Q3_CUDA(e);
  return Q3_OK;
}
extern "C" int q3_set_device(int d) {
  Q3_CUDA(cudaSetDevice(d));
  return Q3_OK;
}
extern "C" int q3_device_info(int d, int* sms, int* ccmaj, int* ccmin, size_t* mem) {
  cudaDeviceProp p;
  Q3_CUDA(cudaGetDeviceProperties(&p, d));
  if (sms) *sms = p.multiProcessorCount;
  if (ccmaj) *ccmaj = p.major;
  if (ccmin) *ccmin = p.minor;
  if (mem) *mem = p.totalGlobalMem;
  return Q3_OK;
}
extern "C" int q3_device_malloc(void** p, size_t n) {
  Q3_REQUIRE(p, "null out pointer");
  cudaError_t e = cudaMalloc(p, n);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    return set_err(Q3_ERR_NOMEM, "cudaMalloc(%zu) failed", n);
  }
  Q3_CUDA(e);
  return Q3_OK;
}
extern "C" int q3_device_free(void* p) {
  Q3_CUDA(cudaFree(p));
  return Q3_OK;
}
extern "C" int q3_host_malloc(void** p, size_t n) {
  Q3_REQUIRE(p, "null out pointer");
  Q3_CUDA(cudaMallocHost(p, n));
  return Q3_OK;
}
extern "C" int q3_host_free(void* p) {
  Q3_CUDA(cudaFreeHost(p));
  return Q3_OK;
}
extern "C" int q3_memcpy_htod(void* d, const void* s, size_t n, void* st) {
  Q3_CUDA(cudaMemcpyAsync(d, s, n, cudaMemcpyHostToDevice, (cudaStream_t)st));
  return Q3_OK;
}
extern "C" int q3_memcpy_dtoh(void* d, const void* s, size_t n, void* st) {
  Q3_CUDA(cudaMemcpyAsync(d, s, n, cudaMemcpyDeviceToHost, (cudaStream_t)st));
  return Q3_OK;
}
extern "C" int q3_memcpy_dtod(void* d, const void* s, size_t n, void* st) {
  Q3_CUDA(cudaMemcpyAsync(d, s, n, cudaMemcpyDeviceToDevice, (cudaStream_t)st));
  return Q3_OK;
}
extern "C" int q3_memset(void* d, int v, size_t n, void* st) {
  Q3_CUDA(cudaMemsetAsync(d, v, n, (cudaStream_t)st));
  return Q3_OK;
}
extern "C" int q3_stream_create(void** s) {
  Q3_REQUIRE(s, "null out pointer");
  cudaStream_t t;
  Q3_CUDA(cudaStreamCreateWithFlags(&t, cudaStreamNonBlocking));
  *s = t;
  return Q3_OK;
}
extern "C" int q3_stream_destroy(void* s) {
  Q3_CUDA(cudaStreamDestroy((cudaStream_t)s));
  return Q3_OK;
}
extern "C" int q3_stream_synchronize(void* s) {
  Q3_CUDA(cudaStreamSynchronize((cudaStream_t)s));
  return Q3_OK;
}
// CUDA graphs of work enqueued on a (non-default) stream, for hosts without
// a CUDA binding that want to replay a sequence of calls.
extern "C" int q3_graph_capture_begin(void* s) {
  Q3_REQUIRE(s, "capture needs a created stream");
  Q3_CUDA(cudaStreamBeginCapture((cudaStream_t)s, cudaStreamCaptureModeThreadLocal));
  return Q3_OK;
}
extern "C" int q3_graph_capture_end(void* s, void** exec) {
  Q3_REQUIRE(s && exec, "null pointer");
  cudaGraph_t g = nullptr;
  Q3_CUDA(cudaStreamEndCapture((cudaStream_t)s, &g));
  cudaGraphExec_t ge = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  Q3_CUDA(e);
  *exec = ge;
  return Q3_OK;
}
extern "C" int q3_graph_launch(void* exec, void* s) {
  Q3_REQUIRE(exec, "null graph");
  Q3_CUDA(cudaGraphLaunch((cudaGraphExec_t)exec, (cudaStream_t)s));
  return Q3_OK;
}
extern "C" int q3_graph_destroy(void* exec) {
  if (exec) Q3_CUDA(cudaGraphExecDestroy((cudaGraphExec_t)exec));
  return Q3_OK;
}
extern "C" int q3_event_create(void** e) {
  Q3_REQUIRE(e, "null out pointer");
  cudaEvent_t t;
  Q3_CUDA(cudaEventCreate(&t));
  *e = t;
  return Q3_OK;
}
extern "C" int q3_event_destroy(void* e) {
  Q3_CUDA(cudaEventDestroy((cudaEvent_t)e));
  return Q3_OK;
}
extern "C" int q3_event_record(void* e, void* s) {
  Q3_CUDA(cudaEventRecord((cudaEvent_t)e, (cudaStream_t)s));
  return Q3_OK;
}
extern "C" int q3_event_synchronize(void* e) {
  Q3_CUDA(cudaEventSynchronize((cudaEvent_t)e));
  return Q3_OK;
}
extern "C" int q3_event_elapsed_ms(void* a, void* b, float* ms) {
  Q3_REQUIRE(ms, "null out pointer");
  Q3_CUDA(cudaEventElapsedTime(ms, (cudaEvent_t)a, (cudaEvent_t)b));
  return Q3_OK;
}

// ---------------------------------------------------------------------------
// host math
// ---------------------------------------------------------------------------
extern "C" int q3_rope_table(int64_t n_pos, float* c, float* s) {
  Q3_REQUIRE(n_pos >= 0 && c && s, "bad rope table arguments");
  for (int64_t p = 0; p < n_pos; ++p) {
    const float pf = (float)(int32_t)p;
    for (int i = 0; i < 64; ++i) {
      const float e = -((2.0f * (float)i) / 128.0f);
      const float th = powf(1.0e6f, e) * 1.0f;
      const float a = pf * th;
      c[p * 64 + i] = cosf(a);
      s[p * 64 + i] = sinf(a);
    }
  }
  return Q3_OK;
}

static void quantize_range(const float* w, uint8_t* out, int64_t b0, int64_t b1) {
  for (int64_t b = b0; b < b1; ++b) {
    const float* blk = w + b * kQBlk;
    float amax = 0.0f;
    for (int j = 0; j < kQBlk; ++j) amax = std::fmax(amax, std::fabs(blk[j]));
    float scale = amax / 127.0f;
    if (scale == 0.0f) scale = 1.0f;
    const __half hs = __float2half_rn(scale);
    uint16_t sh;
    memcpy(&sh, &hs, 2);
    uint8_t* o = out + b * kQBytes;
    o[0] = (uint8_t)(sh & 0xff);
    o[1] = (uint8_t)(sh >> 8);
    for (int j = 0; j < kQBlk; ++j) {
      float q = std::nearbyint(blk[j] / scale);
      q = q < -128.0f ? -128.0f : (q > 127.0f ? 127.0f : q);
      o[2 + j] = (uint8_t)(int8_t)q;
    }
  }
}

extern "C" int q3_quantize_q8_0(const float* w, int64_t n, uint8_t* out) {
  Q3_REQUIRE(w && out && n >= 0 && n % kQBlk == 0, "quantize: n must be a multiple of 32");
  const int64_t nb = n / kQBlk;
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (nb < 65536) nt = 1;
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; ++t)
    th.emplace_back(quantize_range, w, out, nb * t / nt, nb * (t + 1) / nt);
  for (auto& t : th) t.join();
  return Q3_OK;
}

// ---------------------------------------------------------------------------
// launch helpers
// ---------------------------------------------------------------------------
static int current_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 148;
  }
  return cache[dev];
}

constexpr size_t kMaxDynSmem = 200 * 1024;
static std::mutex g_attr_mu;

template <typename F>
static int ensure_smem_attr(F* fn, size_t bytes) {
  // The dynamic shared-memory cap is a per-(kernel, device) attribute; raise it
  // once for each kernel function (keyed by its address) on each device.
  static std::set<std::pair<const void*, int>> done;
  if (bytes <= 48 * 1024) return Q3_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_attr_mu);
  const auto key = std::make_pair((const void*)fn, dev);
  if (done.count(key)) return Q3_OK;
  Q3_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxDynSmem));
  done.insert(key);
  return Q3_OK;
}

// Launch with optional programmatic dependent launch (PDL): the kernel may
// begin while the previous kernel in the stream finishes; kernels call
// griddepcontrol.wait before touching that kernel's outputs.
template <typename... KArgs, typename... Args>
static cudaError_t launch_ex(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// The same with thread-block clusters of cluster_y CTAs along y.
template <typename... KArgs, typename... Args>
static cudaError_t launch_cluster(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t st, bool pdl, int cluster_y, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = 1;
  attr[n].val.clusterDim.y = (unsigned)cluster_y;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// The same with clusters of cluster_x CTAs along x (sizes above 8 need the
// kernel's non-portable cluster attribute).
template <typename... KArgs, typename... Args>
static cudaError_t launch_cluster_x(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t st, bool pdl, int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = (unsigned)cluster_x;
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// Tensor maps are encoded through the driver entry point
// cuTensorMapEncodeTiled (no link-time libcuda dependency).
typedef CUresult (*PfnEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PfnEncodeTiled encode_fn() {
  static PfnEncodeTiled fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PfnEncodeTiled)p;
  }
  return fn;
}

// 2-D map over a row-major matrix: `inner` elements per row, `outer` rows,
// rows `row_bytes` apart; box {box_inner, box_outer}.
static int make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                       uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                       CUtensorMapSwizzle sw) {
  PfnEncodeTiled fn = encode_fn();
  if (!fn) return set_err(Q3_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  Q3_REQUIRE(((uintptr_t)base & 15u) == 0 && row_bytes % 16 == 0,
             "tensor map base / row stride must be 16-byte aligned");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_err(Q3_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q3_OK;
}

struct LaunchShape {
  int grid, nstages;
  size_t smem;
};

// Tiles at or below this many per SM run one tile per CTA (Q3_GEMV_ONE_TILE_PER_SM overrides).
static int one_tile_threshold() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("Q3_GEMV_ONE_TILE_PER_SM");
    const int x = e ? atoi(e) : 0;
    v = (x >= 1 && x <= 16) ? x : 4;
  }
  return v;
}

// CTAs per SM of a multi-tile Q8_0 GEMV launch: 3 (measured over 28-layer
// launches: 2.2-3.2 TB/s against 2.0-3.0 at 2); Q3_GEMV_STREAM_CTAS overrides, 1..4.
static int gemv_stream_ctas() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("Q3_GEMV_STREAM_CTAS");
    const int x = e ? atoi(e) : 0;
    v = (x >= 1 && x <= 4) ? x : 3;
  }
  return v;
}

// Shared memory of one SM and the part of it each CTA loses to the runtime.
static void sm_smem_limits(size_t* per_sm, size_t* reserved) {
  int dev = 0, v = 0, r = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess)
    v = 0;
  if (cudaDeviceGetAttribute(&r, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess)
    r = 1024;
  *per_sm = v > 0 ? (size_t)v : 228 * 1024;
  *reserved = (size_t)r;
}

// Grid and ring depth: one tile per CTA for small launches, else
// ctas_per_sm_stream CTAs on every SM, each ring as deep as the SM's shared
// memory allows once every CTA's static shared memory (static_smem) and
// reservation are counted.
static LaunchShape stream_shape(int ntiles, uint32_t tile_bytes, int ctas_per_sm_stream,
                                size_t static_smem = 0) {
  const int sms = current_sms();
  LaunchShape s;
  if (ntiles <= one_tile_threshold() * sms) {
    s.grid = ntiles > 0 ? ntiles : 1;
    s.nstages = 1;
  } else {
    s.grid = ctas_per_sm_stream * sms;
    const int tpc = (ntiles + s.grid - 1) / s.grid;
    size_t budget = (size_t)(kMaxDynSmem / ctas_per_sm_stream) - 1024;
    if (static_smem > 0) {
      size_t per_sm = 0, reserved = 0;
      sm_smem_limits(&per_sm, &reserved);
      const size_t share = per_sm / ctas_per_sm_stream;
      const size_t fit = share > reserved + static_smem + 256 ? share - reserved - static_smem - 256 : 0;
      budget = std::min(budget, fit);
    }
    int ns = (int)(budget / tile_bytes);
    if (ns < 1) ns = 1;
    if (ns > 16) ns = 16;
    if (ns > tpc) ns = tpc;
    s.nstages = ns;
  }
  s.smem = ring_smem_bytes(s.nstages, tile_bytes);
  return s;
}

template <int G, int ORDER, int MODE>
static int launch_q8_t(Q8GemvArgs a, cudaStream_t st, int* launches, bool pdl) {
  const uint32_t rowbytes = (uint32_t)(a.K / kQBlk) * kQBytes;
  const uint32_t tile_bytes = rowbytes * kTileRows * (MODE == kModeSwiglu ? 2u : 1u);
  const int ntiles = a.nseg * (a.seg_rows / kTileRows);
  if (ntiles <= one_tile_threshold() * current_sms()) {
    // one tile per CTA: weights converted to registers before the dependency wait
    int rc = ensure_smem_attr(k_gemv_q8_1t<G, ORDER, MODE>, tile_bytes);
    if (rc) return rc;
    Q3_CUDA(launch_ex(k_gemv_q8_1t<G, ORDER, MODE>, dim3(ntiles > 0 ? ntiles : 1),
                      dim3(kGemv1tThreads), (size_t)tile_bytes, st, pdl, a));
    if (launches) ++*launches;
    return Q3_OK;
  }
  static size_t static_smem = 0;
  if (static_smem == 0) {
    cudaFuncAttributes fa;
    static_smem = cudaFuncGetAttributes(&fa, k_gemv_q8<G, ORDER, MODE>) == cudaSuccess
                      ? fa.sharedSizeBytes + 16
                      : 16 * 1024;
  }
  LaunchShape ls = stream_shape(ntiles, tile_bytes, gemv_stream_ctas(), static_smem);
  a.nstages = ls.nstages;
  int rc = ensure_smem_attr(k_gemv_q8<G, ORDER, MODE>, ls.smem);
  if (rc) return rc;
  Q3_CUDA(launch_ex(k_gemv_q8<G, ORDER, MODE>, dim3(ls.grid), dim3(kGemvThreads), ls.smem, st, pdl,
                    a));
  if (launches) ++*launches;
  return Q3_OK;
}

template <int ORDER, int MODE>
static int launch_q8(const Q8GemvArgs& a, cudaStream_t st, int* launches, bool pdl = false) {
  switch ((a.K + 1023) / 1024) {
    case 1: return launch_q8_t<1, ORDER, MODE>(a, st, launches, pdl);
    case 2: return launch_q8_t<2, ORDER, MODE>(a, st, launches, pdl);
    case 3: return launch_q8_t<3, ORDER, MODE>(a, st, launches, pdl);
    default: return set_err(Q3_ERR_UNSUPPORTED, "K=%d above 3072", a.K);
  }
}

static int check_q8_shape(const void* w, const void* x, const void* y, int N, int K) {
  Q3_REQUIRE(w && x && y, "null pointer");
  Q3_REQUIRE(K > 0 && K % 256 == 0 && K <= 3072, "K=%d must be a multiple of 256, <= 3072", K);
  Q3_REQUIRE(N > 0 && N % 8 == 0, "N=%d must be a positive multiple of 8", N);
  Q3_REQUIRE(aligned16(w) && aligned16(x), "w and x must be 16-byte aligned");
  return Q3_OK;
}

static Q8GemvArgs q8_args_single(const void* w, const void* x, void* y, const void* r, int N,
                                 int K) {
  Q8GemvArgs a;
  memset(&a, 0, sizeof(a));
  a.seg[0].w = (const uint8_t*)w;
  a.seg[0].x = (const uint16_t*)x;
  a.seg[0].y = (uint16_t*)y;
  a.seg[0].r = (const uint16_t*)r;
  a.nseg = 1;
  a.seg_rows = N;
  a.K = K;
  return a;
}

extern "C" int q3_gemv_q8(const void* w, const void* x, void* y, int N, int K, void* stream) {
  int rc = check_q8_shape(w, x, y, N, K);
  if (rc) return rc;
  return launch_q8<kOrderMlir, kModePlain>(q8_args_single(w, x, y, nullptr, N, K),
                                          (cudaStream_t)stream, nullptr);
}

extern "C" int q3_gemv_q8_overlapped(const void* w, const void* x, void* y, int N, int K,
                                     void* stream) {
  int rc = check_q8_shape(w, x, y, N, K);
  if (rc) return rc;
  return launch_q8<kOrderMlir, kModePlain>(q8_args_single(w, x, y, nullptr, N, K),
                                          (cudaStream_t)stream, nullptr, true);
}

extern "C" int q3_gemv_q8_cuda_order(const void* w, const void* x, void* y, int N, int K,
                                     void* stream) {
  int rc = check_q8_shape(w, x, y, N, K);
  if (rc) return rc;
  return launch_q8<kOrderCuda, kModePlain>(q8_args_single(w, x, y, nullptr, N, K),
                                          (cudaStream_t)stream, nullptr);
}

extern "C" int q3_gemv_q8_layers(const void* w, int64_t w_stride, const void* x, void* y, int N,
                                 int K, int L, void* stream) {
  int rc = check_q8_shape(w, x, y, N, K);
  if (rc) return rc;
  Q3_REQUIRE(L >= 1 && L <= kMaxSeg, "L=%d must be in [1, %d]", L, kMaxSeg);
  Q3_REQUIRE(w_stride % 16 == 0, "w_stride must be a multiple of 16");
  Q8GemvArgs a = q8_args_single(w, x, y, nullptr, N, K);
  a.nseg = L;
  for (int l = 0; l < L; ++l) {
    a.seg[l].w = (const uint8_t*)w + (int64_t)l * w_stride;
    a.seg[l].x = (const uint16_t*)x + (int64_t)l * K;
    a.seg[l].y = (uint16_t*)y + (int64_t)l * N;
  }
  return launch_q8<kOrderMlir, kModePlain>(a, (cudaStream_t)stream, nullptr);
}

extern "C" int q3_gemv_q8_norm(const void* w, const void* x, const void* gamma, void* y, int N,
                               int K, void* stream) {
  int rc = check_q8_shape(w, x, y, N, K);
  if (rc) return rc;
  Q3_REQUIRE(gamma, "gamma is null");
  Q8GemvArgs a = q8_args_single(w, x, y, nullptr, N, K);
  a.norm_g = (const uint16_t*)gamma;
  return launch_q8<kOrderMlir, kModeNormIn>(a, (cudaStream_t)stream, nullptr);
}

extern "C" int q3_gemv_q8_resid(const void* w, const void* x, const void* r, void* y, int N,
                                int K, void* stream) {
  int rc = check_q8_shape(w, x, y, N, K);
  if (rc) return rc;
  Q3_REQUIRE(r, "r is null");
  return launch_q8<kOrderMlir, kModeResid>(q8_args_single(w, x, y, r, N, K),
                                          (cudaStream_t)stream, nullptr);
}

extern "C" int q3_gemv_q8_swiglu(const void* w, const void* x, const void* gamma, void* y, int N,
                                 int K, void* stream) {
  int rc = check_q8_shape(w, x, y, N, K);
  if (rc) return rc;
  Q3_REQUIRE(gamma, "gamma is null");
  Q8GemvArgs a = q8_args_single(w, x, y, nullptr, N, K);
  a.norm_g = (const uint16_t*)gamma;
  a.up_off_bytes = (int64_t)N * (K / kQBlk) * kQBytes;
  return launch_q8<kOrderMlir, kModeSwiglu>(a, (cudaStream_t)stream, nullptr);
}

// vocab + argmax ------------------------------------------------------------
constexpr int kArgmaxMaxGrid = 4096;
extern "C" size_t q3_vocab_argmax_workspace_bytes(void) {
  return sizeof(ArgmaxPartial) * kArgmaxMaxGrid + 256;
}

static int launch_vocab(VocabArgs a, cudaStream_t st, int* launches, bool pdl = false) {
  const uint32_t tile_bytes = (uint32_t)a.K * 2u * kTileRows;
  LaunchShape ls = stream_shape(a.N / kTileRows, tile_bytes, 2);
  if (ls.grid > kArgmaxMaxGrid) ls.grid = kArgmaxMaxGrid;
  a.nstages = ls.nstages;
  int rc = ensure_smem_attr(k_vocab_argmax, ls.smem);
  if (rc) return rc;
  Q3_CUDA(launch_ex(k_vocab_argmax, dim3(ls.grid), dim3(kGemvThreads), ls.smem, st, pdl, a));
  if (launches) ++*launches;
  return Q3_OK;
}

extern "C" int q3_vocab_argmax(const void* w, const void* x, const void* gamma, void* logits,
                               int64_t* token, void* ws, int N, int K, void* stream) {
  Q3_REQUIRE(w && x && token && ws, "null pointer");
  Q3_REQUIRE(K == kVocabK, "K=%d: this build covers K == 1024", K);
  Q3_REQUIRE(N > 0 && N % 8 == 0, "N=%d must be a positive multiple of 8", N);
  Q3_REQUIRE(aligned16(w) && aligned16(ws), "w and workspace must be 16-byte aligned");
  VocabArgs a;
  memset(&a, 0, sizeof(a));
  a.w = (const uint16_t*)w;
  a.x = (const uint16_t*)x;
  a.norm_g = (const uint16_t*)gamma;
  a.logits = (uint16_t*)logits;
  a.N = N;
  a.K = K;
  a.partial = (ArgmaxPartial*)ws;
  a.counter = (unsigned int*)((uint8_t*)ws + sizeof(ArgmaxPartial) * kArgmaxMaxGrid);
  a.token_out = token;
  return launch_vocab(a, (cudaStream_t)stream, nullptr);
}

// attention -----------------------------------------------------------------
// Chunks of 32 keys a cache of S positions can hold, and 8-chunk groups.
static int max_chunks_for(int64_t S) { return (int)((S + kAttChunk - 1) / kAttChunk); }
static int max_groups_for(int64_t S) {
  return (max_chunks_for(S) + kAttSplitChunks - 1) / kAttSplitChunks;
}

extern "C" size_t q3_attention_workspace_bytes(int64_t S) {
  const int mc = max_chunks_for(S < 1 ? 1 : S);
  return sizeof(AttnPartial) * (size_t)kNKV * mc * 2 + 256;
}

// K/V loads issued before the norms (1 CTA per SM at 182 registers) or after
// them (2 CTAs per SM); Q3_ATTN_EARLY=0|1 overrides the per-batch default.
static bool attn_early_loads(int batch) {
  static int env = -2;
  if (env == -2) {
    const char* e = getenv("Q3_ATTN_EARLY");
    env = (e && (e[0] == '0' || e[0] == '1')) ? e[0] - '0' : -1;
  }
  if (env >= 0) return env == 1;
  return batch == 1;
}

// groups > 0 sizes the grid's group dimension below the partial stride
// (a.max_chunks), for a scratch laid out for longer caches than this launch's.
static int launch_attn(const AttnArgs& a, int batch, cudaStream_t st, int* launches,
                       bool pdl = false, int groups = 0) {
  if (groups <= 0) groups = max_groups_for((int64_t)a.max_chunks * kAttChunk);
  dim3 grid(kNKV, (unsigned)groups, batch);
  if (attn_early_loads(batch))
    Q3_CUDA(launch_ex(k_attn_decode<true>, grid, dim3(256), 0, st, pdl, a));
  else
    Q3_CUDA(launch_ex(k_attn_decode<false>, grid, dim3(256), 0, st, pdl, a));
  if (launches) ++*launches;
  return Q3_OK;
}

extern "C" int q3_decode_attention(const void* qkv, const void* q_norm, const void* k_norm,
                                   const float* rope_cos, const float* rope_sin, int64_t rope_rows,
                                   void* kc, void* vc, int64_t slot0, int64_t S, const int64_t* pos,
                                   void* out, void* ws, void* stream) {
  Q3_REQUIRE(qkv && q_norm && k_norm && rope_cos && rope_sin && kc && vc && pos && out && ws,
             "null pointer");
  Q3_REQUIRE(S >= 1 && slot0 >= 0 && rope_rows >= 1, "bad S / slot0 / rope_rows");
  Q3_REQUIRE(aligned16(qkv) && aligned16(kc) && aligned16(vc) && aligned16(ws),
             "qkv, caches and workspace must be 16-byte aligned");
  Q3_REQUIRE(((uintptr_t)out & 7u) == 0, "out must be 8-byte aligned (stored as 4 f16 at a time)");
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.qkv = (const uint16_t*)qkv;
  a.q_norm = (const uint16_t*)q_norm;
  a.k_norm = (const uint16_t*)k_norm;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.rope_pos = rope_rows;
  a.kc = (uint16_t*)kc;
  a.vc = (uint16_t*)vc;
  a.slot0 = slot0;
  a.S = S;
  a.pos = pos;
  a.pos_stride = 1;
  a.out = (uint16_t*)out;
  a.max_chunks = max_chunks_for(S);
  a.part = (AttnPartial*)ws;
  a.counters = (unsigned int*)((uint8_t*)ws + sizeof(AttnPartial) * (size_t)kNKV * a.max_chunks * 2);
  return launch_attn(a, 1, (cudaStream_t)stream, nullptr);
}

// Attention with no caller workspace -------------------------------------------
// Some callers cannot allocate device memory at the point where they launch:
// a kernel substituted into an IREE executable receives only its bindings and
// push constants (the HAL allocates nothing on its behalf), and code that
// runs inside a fixed memory plan must not call cudaMalloc.  For them this
// entry point keeps the attention kernel's scratch (the per-chunk softmax
// partials and the per-head arrival counters) in one file-scope device array
// sized for contexts of up to kNoAllocMaxPositions positions (1,081,600
// bytes; every device that loads this library holds it until process exit).
constexpr int64_t kNoAllocMaxPositions = 4096;
constexpr int kNoAllocChunks = (int)(kNoAllocMaxPositions / kAttChunk);
constexpr size_t kNoAllocPartBytes = sizeof(AttnPartial) * (size_t)kNKV * kNoAllocChunks * 2;
static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocPartBytes + 256];

// Device address of g_attn_scratch per device.  In host code the symbol is a
// host-side stand-in, never a device address; the address comes from
// cudaGetSymbolAddress, taken once per device with that device current.
static std::mutex g_scratch_mu;
static void* g_scratch_addr[64] = {nullptr};

extern "C" int q3_decode_attention_noalloc(const void* qkv, const void* q_norm, const void* k_norm,
                                           const float* rope_cos, const float* rope_sin,
                                           int64_t rope_rows, void* kc, void* vc, int64_t slot0,
                                           int64_t S, const int64_t* pos, void* out,
                                           void* stream) {
  Q3_REQUIRE(qkv && q_norm && k_norm && rope_cos && rope_sin && kc && vc && pos && out,
             "null pointer");
  Q3_REQUIRE(S >= 1 && slot0 >= 0 && rope_rows >= 1, "bad S / slot0 / rope_rows");
  Q3_REQUIRE(S <= kNoAllocMaxPositions,
             "S=%lld exceeds the %lld positions the static attention scratch holds; use "
             "q3_decode_attention with a workspace",
             (long long)S, (long long)kNoAllocMaxPositions);
  Q3_REQUIRE(aligned16(qkv) && aligned16(kc) && aligned16(vc),
             "qkv and caches must be 16-byte aligned");
  Q3_REQUIRE(((uintptr_t)out & 7u) == 0, "out must be 8-byte aligned (stored as 4 f16 at a time)");
  int dev = 0;
  Q3_CUDA(cudaGetDevice(&dev));
  Q3_REQUIRE(dev >= 0 && dev < 64, "device ordinal %d out of range", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch_addr[dev] == nullptr) {
      void* p = nullptr;
      Q3_CUDA(cudaGetSymbolAddress(&p, g_attn_scratch));
      g_scratch_addr[dev] = p;
    }
    scratch = g_scratch_addr[dev];
  }
  unsigned int* counters = (unsigned int*)((uint8_t*)scratch + kNoAllocPartBytes);
  // the counters must start at zero; the partials are written before they are read
  Q3_CUDA(cudaMemsetAsync(counters, 0, kNKV * sizeof(unsigned int), (cudaStream_t)stream));
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.qkv = (const uint16_t*)qkv;
  a.q_norm = (const uint16_t*)q_norm;
  a.k_norm = (const uint16_t*)k_norm;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.rope_pos = rope_rows;
  a.kc = (uint16_t*)kc;
  a.vc = (uint16_t*)vc;
  a.slot0 = slot0;
  a.S = S;
  a.pos = pos;
  a.pos_stride = 1;
  a.out = (uint16_t*)out;
  a.max_chunks = kNoAllocChunks;
  a.part = (AttnPartial*)scratch;
  a.counters = counters;
  // partials keep the scratch's stride; the grid covers only this cache's groups
  return launch_attn(a, 1, (cudaStream_t)stream, nullptr, false, max_groups_for(S));
}

// One layer of the fused engine on caller buffers ------------------------------
// Tensor maps of the fused kernels: W_o and W_down of all layers as u32
// matrices (boxes: a head pair's 272-byte slice of 64 rows; a slice's
// 416-byte window of 64 rows), the K cache (64-dim half boxes, 128-byte
// swizzle) and the V cache of `slots` positions.
struct FusedMaps {
  CUtensorMap wo, k, v, wd;
};

static int make_fused_maps(FusedMaps* f, const q3_weights* w, const void* kc, const void* vc,
                           int64_t slots) {
  int rc = make_map_2d(&f->wo, CU_TENSOR_MAP_DATA_TYPE_UINT32, w->q8_attn_output, kORowBytes / 4,
                       (uint64_t)kLayers * kDim, kORowBytes, kFaOBytes / 4, kFaORows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == Q3_OK)
    rc = make_map_2d(&f->k, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, kc, (uint64_t)kNKV * kHD,
                     (uint64_t)slots, (uint64_t)kNKV * kHD * 2, 64, kFaChunk,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == Q3_OK)
    rc = make_map_2d(&f->v, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, vc, (uint64_t)kNKV * kHD,
                     (uint64_t)slots, (uint64_t)kNKV * kHD * 2, kHD, kFaChunk,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc == Q3_OK)
    rc = make_map_2d(&f->wd, CU_TENSOR_MAP_DATA_TYPE_UINT32, w->q8_ffn_down, kDRowBytes / 4,
                     (uint64_t)kLayers * kDim, kDRowBytes, kFbDWin / 4, kFbDRows,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
  return rc;
}

// The fused kernels' attributes (dynamic shared memory above 48 KB, 16-CTA
// clusters), set once per device.
static int fused_attrs() {
  static std::mutex mu;
  static std::set<int> done;
  int dev = 0;
  Q3_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done.count(dev)) return Q3_OK;
  Q3_CUDA(cudaFuncSetAttribute(k_fused_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFaSmem));
  Q3_CUDA(cudaFuncSetAttribute(k_fused_attn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  Q3_CUDA(cudaFuncSetAttribute(k_fused_ffn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFbSmem));
  Q3_CUDA(cudaFuncSetAttribute(k_fused_ffn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  // One carve-out for every kernel of the step: an SM configured for one of
  // them can then take a CTA of the next one beside it.
  Q3_CUDA(cudaFuncSetAttribute(k_fused_attn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared));
  Q3_CUDA(cudaFuncSetAttribute(k_fused_ffn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared));
  Q3_CUDA(cudaFuncSetAttribute(k_vocab_argmax, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared));
  done.insert(dev);
  return Q3_OK;
}

// Workspace: the O and down partials, h1 and the intermediate x.
struct FusedLayerWs {
  float opart[kFParts * kDim];
  float dpart[kFParts * kDim];
  uint16_t x[kDim];
  uint16_t h1[kDim];
};

extern "C" size_t q3_fused_layer_workspace_bytes(void) { return sizeof(FusedLayerWs) + 256; }

extern "C" int q3_fused_layer(const q3_weights* w, int layer, const void* x_in, void* x_out,
                              void* kc, void* vc, int64_t S, const int64_t* pos,
                              const float* rope_cos, const float* rope_sin, void* ws, int flags,
                              void* stream) {
  Q3_REQUIRE(w && x_in && x_out && kc && vc && pos && rope_cos && rope_sin && ws, "null pointer");
  Q3_REQUIRE(layer >= 0 && layer < kLayers, "layer %d out of range", layer);
  Q3_REQUIRE(S >= 1 && S <= kFusedMaxPositions, "S=%lld outside [1, %lld]", (long long)S,
             (long long)kFusedMaxPositions);
  Q3_REQUIRE(aligned16(x_in) && aligned16(x_out) && aligned16(kc) && aligned16(vc) && aligned16(ws),
             "x, caches and workspace must be 16-byte aligned");
  const void* req[] = {w->attn_norm, w->ffn_norm, w->attn_q_norm, w->attn_k_norm, w->q8_attn_q,
                       w->q8_attn_k, w->q8_attn_v, w->q8_attn_output, w->q8_ffn_gate_up,
                       w->q8_ffn_down};
  for (const void* p : req) Q3_REQUIRE(p != nullptr && aligned16(p), "weights: null or unaligned");
  int rc_ = Q3_OK;
  cudaStream_t st = (cudaStream_t)stream;
  FusedLayerWs* f = (FusedLayerWs*)ws;
  FusedMaps maps;
  Q3_REQUIRE((flags & ~Q3_LAYER_OVERLAP) == 0, "unknown flags 0x%x", flags);
  rc_ = make_fused_maps(&maps, w, kc, vc, (int64_t)(layer + 1) * S);
  if (rc_) return rc_;
  rc_ = fused_attrs();
  if (rc_) return rc_;
  FaArgs fa;
  memset(&fa, 0, sizeof(fa));
  fa.wq = (const uint8_t*)w->q8_attn_q + layer * kBplQ;
  fa.wk = (const uint8_t*)w->q8_attn_k + layer * kBplKV;
  fa.wv = (const uint8_t*)w->q8_attn_v + layer * kBplKV;
  fa.wo_map = maps.wo;
  fa.k_map = maps.k;
  fa.v_map = maps.v;
  fa.layer = layer;
  fa.attn_norm = (const uint16_t*)w->attn_norm + layer * kDim;
  fa.q_norm = (const uint16_t*)w->attn_q_norm + layer * kHD;
  fa.k_norm = (const uint16_t*)w->attn_k_norm + layer * kHD;
  fa.h1 = (const uint16_t*)x_in;  // no dpart: x = x_in
  fa.x_out = f->x;
  fa.opart = f->opart;
  fa.kc = (uint16_t*)kc;
  fa.vc = (uint16_t*)vc;
  fa.rope_cos = rope_cos;
  fa.rope_sin = rope_sin;
  fa.slot0 = (int64_t)layer * S;
  fa.S = S;
  fa.pos = pos;
  Q3_CUDA(launch_cluster_x(k_fused_attn, dim3(kFParts * kFC), dim3(kFaThreads), kFaSmem, st,
                           (flags & Q3_LAYER_OVERLAP) != 0, kFC, fa));
  FbArgs fb;
  memset(&fb, 0, sizeof(fb));
  fb.wgu = (const uint8_t*)w->q8_ffn_gate_up + layer * kBplGU;
  fb.wd_map = maps.wd;
  fb.layer = layer;
  fb.ffn_norm = (const uint16_t*)w->ffn_norm + layer * kDim;
  fb.x = f->x;
  fb.opart = f->opart;
  fb.h1_out = f->h1;
  fb.dpart = f->dpart;
  Q3_CUDA(launch_cluster_x(k_fused_ffn, dim3(kFParts * kFC), dim3(kFbThreads), kFbSmem, st, true,
                           kFC, fb));
  Q3_CUDA(launch_ex(k_resid_parts, dim3(1), dim3(256), 0, st, true, (const uint16_t*)f->h1,
                    (const float*)f->dpart, (uint16_t*)x_out));
  return Q3_OK;
}

// Error-path plumbing ---------------------------------------------------------
// One thread waits, bounded by limit_cycles of SM clock, for *flag == expect;
// on expiry it records kErrTimeoutGrid in *err (the same bounded-wait pattern
// as every wait of the decode kernels) and returns, leaving the context usable.
__global__ void k_bounded_wait(const int* flag, int expect, long long limit, int* err) {
  if (threadIdx.x != 0) return;
  const long long t0 = clock64();
  while (*(volatile const int*)flag != expect) {
    if (clock64() - t0 > limit) {
      atomicCAS(err, 0, kErrTimeoutGrid);
      return;
    }
  }
}

extern "C" int q3_selftest_bounded_wait(const int* flag, int expect, int64_t limit_cycles,
                                        int* err, void* stream) {
  Q3_REQUIRE(flag && err, "null pointer");
  Q3_REQUIRE(limit_cycles >= 1 && limit_cycles <= kSpinCycles,
             "limit_cycles must be in [1, %lld]", (long long)kSpinCycles);
  k_bounded_wait<<<1, 32, 0, (cudaStream_t)stream>>>(flag, expect, (long long)limit_cycles, err);
  Q3_CUDA(cudaGetLastError());
  return Q3_OK;
}

extern "C" int q3_check_error_word(const int* err, void* stream) {
  Q3_REQUIRE(err, "null pointer");
  int code = 0;
  Q3_CUDA(cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  Q3_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  if (code != 0) return set_err(Q3_ERR_DEVICE, "kernel error word %d", code);
  return Q3_OK;
}

// IREE-ABI dispatch launchers --------------------------------------------------
#define Q3_IREE_CHECK(w, b1, b2)                                                  \
  Q3_REQUIRE((w) && (b1) && (b2), "null binding");                                \
  Q3_REQUIRE(aligned16(w) && aligned16(b1), "bindings 0 and 1 must be 16-byte aligned")

extern "C" int q3_iree_dispatch_3(const void* q8, const void* b1, void* b2, uint32_t c0,
                                  uint32_t c1, void* stream) {
  Q3_IREE_CHECK(q8, b1, b2);
  decode_dispatch_3_matmul_2048x1x1024_f16<<<256, 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)q8, (const char*)b1, (char*)b2, c0, c1);
  Q3_LAUNCHED();
  return Q3_OK;
}
extern "C" int q3_iree_dispatch_4(const void* q8, const void* b1, void* b2, uint32_t c0,
                                  uint32_t c1, uint32_t c2, void* stream) {
  Q3_IREE_CHECK(q8, b1, b2);
  decode_dispatch_4_matmul_1024x1x1024_f16<<<128, 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)q8, (const char*)b1, (char*)b2, c0, c1, c2);
  Q3_LAUNCHED();
  return Q3_OK;
}
extern "C" int q3_iree_dispatch_12(const void* q8, const void* b1, void* b2, uint32_t c0,
                                   uint32_t c1, void* stream) {
  Q3_IREE_CHECK(q8, b1, b2);
  decode_dispatch_12_matmul_1024x1x2048_f16<<<128, 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)q8, (const char*)b1, (char*)b2, c0, c1);
  Q3_LAUNCHED();
  return Q3_OK;
}
extern "C" int q3_iree_dispatch_18(const void* q8, const void* b1, void* b2, uint32_t c0,
                                   uint32_t c1, void* stream) {
  Q3_IREE_CHECK(q8, b1, b2);
  decode_dispatch_18_matmul_6144x1x1024_f16<<<768, 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)q8, (const char*)b1, (char*)b2, c0, c1);
  Q3_LAUNCHED();
  return Q3_OK;
}
extern "C" int q3_iree_dispatch_20(const void* q8, const void* b1, void* b2, uint32_t c0,
                                   uint32_t c1, void* stream) {
  Q3_IREE_CHECK(q8, b1, b2);
  decode_dispatch_20_matmul_1024x1x3072_f16<<<128, 256, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)q8, (const char*)b1, (char*)b2, c0, c1);
  Q3_LAUNCHED();
  return Q3_OK;
}
extern "C" int q3_iree_dispatch_24(const void* w, const void* b1, void* b2, uint32_t c0,
                                   void* stream) {
  Q3_IREE_CHECK(w, b1, b2);
  decode_dispatch_24_matmul_151936x1x1024_f16<<<18992, 256, 0, (cudaStream_t)stream>>>(
      (const __half*)w, (const char*)b1, (char*)b2, c0);
  Q3_LAUNCHED();
  return Q3_OK;
}

// ---------------------------------------------------------------------------
// decoder object
// ---------------------------------------------------------------------------
struct q3_model {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  q3_weights w{};
  int64_t S = 0;
  // owned device memory
  uint16_t *kc = nullptr, *vc = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  uint16_t *x = nullptr, *qkv = nullptr, *attn = nullptr, *h1 = nullptr, *act = nullptr,
           *logits = nullptr;
  int64_t* tokens = nullptr;  // [S + 1]: token at each position
  SeqState* st = nullptr;
  ArgmaxPartial* am_part = nullptr;
  unsigned int* am_counter = nullptr;
  AttnPartial* att_part = nullptr;
  unsigned int* att_counters = nullptr;
  int* err = nullptr;
  // pinned host staging
  SeqState* h_st = nullptr;
  int64_t* h_tokens = nullptr;
  // graphs
  cudaGraphExec_t g_ingest = nullptr, g_gen = nullptr, g_prof = nullptr;
  int launches_gen = 0, launches_ingest = 0;
  std::vector<cudaEvent_t> prof_events;
  std::vector<int32_t> prof_kinds;
  // generation bookkeeping
  int64_t gen_n_prompt = 0, gen_pos0 = 0, gen_max = 0;
  bool gen_active = false;
  // chat
  // engines: CUDA graphs of per-phase kernels (exact: 5 per layer; fused: 2
  // cluster kernels per layer), or one persistent kernel
  int engine = Q3_ENGINE_GRAPH;
  float *opart = nullptr, *dpart = nullptr;  // fused engine: split O / down partials [8][1024]
  struct FusedMaps* fmaps = nullptr;         // fused engine: tensor maps (weights, caches)
  cudaGraphExec_t g_ingest_f = nullptr, g_gen_f = nullptr;
  int launches_gen_f = 0, launches_ingest_f = 0;
  int fused_clusters = 0;        // co-resident 16-CTA clusters of the fused kernels (0: unavailable)
  int prof_engine = -1, ktrace_engine = -1;  // engine the profiling graphs were captured for
  int persist_grid = 0;          // CTAs of the persistent kernel (one per SM)
  unsigned int* grid_ctr = nullptr;
  int64_t kernel_launches = 0;   // kernels launched by this model so far
  long long* trace_dev = nullptr; // persistent-kernel phase trace (when tracing)
  cudaGraphExec_t g_ktrace = nullptr;     // graph-engine step with launch timing records
  unsigned long long* ktrace_dev = nullptr;
  std::vector<int32_t> ktrace_kinds;
  int trace_step = -1;
  bool chat_ready = false;
  int64_t chat_pos = 0, chat_max = 0;
  int prefill_mode = Q3_PREFILL_STEPS;  // how prompts are ingested
  q3_batch* pf = nullptr;               // prefill view (batched kernels on this model's cache)
};

// Prompt prefill through the batched kernels (defined with the batched decoder).
static int model_prefill(q3_model* m, int64_t pos0, int64_t n);
static void prefill_destroy(q3_batch* pf);

// Optional instrumentation while capturing: after every kernel an event is
// recorded and the kernel's kind appended (profiling graph only).
struct StepProbe {
  std::vector<cudaEvent_t>* events = nullptr;
  std::vector<int32_t>* kinds = nullptr;
  unsigned long long* ktrace = nullptr;  // launch timing records, kTraceVals per kernel
  int* slot = nullptr;                   // next record
  std::vector<int32_t>* tkinds = nullptr;
  long long* phase = nullptr;            // fused kernels' per-CTA phase stamps, per launch
  int* pslot = nullptr;
  long long* bphase = nullptr;           // batched kernels' per-CTA phase stamps, per launch
  std::vector<int32_t>* bkinds = nullptr;
};

// The next fused launch's phase-stamp block while capturing a phase-traced graph.
static long long* probe_phase(const StepProbe* pr) {
  if (!pr || !pr->phase) return nullptr;
  return pr->phase + (int64_t)kFParts * kFC * kFPhases * (*pr->pslot)++;
}

// The next launch's timing record while capturing a traced graph, else null.
static unsigned long long* probe_trace(const StepProbe* pr, int kind) {
  if (!pr || !pr->ktrace) return nullptr;
  pr->tkinds->push_back(kind);
  return pr->ktrace + kTraceVals * (*pr->slot)++;
}

static int probe_mark(const StepProbe* pr, cudaStream_t st, int kind) {
  if (!pr || !pr->events) return Q3_OK;
  cudaEvent_t e;
  Q3_CUDA(cudaEventCreate(&e));
  pr->events->push_back(e);
  pr->kinds->push_back(kind);
  Q3_CUDA(cudaEventRecordWithFlags(e, st, cudaEventRecordExternal));
  return Q3_OK;
}

#define Q3_PROBE(kind)                          \
  do {                                          \
    int rc_ = probe_mark(probe, st, (kind));    \
    if (rc_) return rc_;                        \
  } while (0)

// Each Q8_0 launch of a step prefetches the next Q8_0 launch's weights into
// L2 (Q3_GEMV_L2_PREFETCH=0 turns it off, for measurement).
static bool gemv_l2_prefetch() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("Q3_GEMV_L2_PREFETCH");
    v = (e && atoi(e) == 0) ? 0 : 1;
  }
  return v != 0;
}

static void set_prefetch(Q8GemvArgs& a, int r, const void* p, int64_t bytes) {
  if (!gemv_l2_prefetch()) return;
  a.pf_ptr[r] = (const uint8_t*)p;
  a.pf_bytes[r] = (uint32_t)bytes;
}

static int enqueue_layers(q3_model* m, bool ingest, int* launches, const StepProbe* probe) {
  cudaStream_t st = m->stream;
  const int32_t* stop = &m->st->stop;
  for (int l = 0; l < kLayers; ++l) {
    // 1) RMSNorm + Q|K|V projections (layer 0 also gathers the embedding)
    Q8GemvArgs a;
    memset(&a, 0, sizeof(a));
    const uint8_t* wq = (const uint8_t*)m->w.q8_attn_q + l * kBplQ;
    const uint8_t* wk = (const uint8_t*)m->w.q8_attn_k + l * kBplKV;
    const uint8_t* wv = (const uint8_t*)m->w.q8_attn_v + l * kBplKV;
    const int64_t rb = 1088;
    a.seg[0] = {wq, m->x, m->qkv, nullptr};
    a.seg[1] = {wq + 1024 * rb, m->x, m->qkv + 1024, nullptr};
    a.seg[2] = {wk, m->x, m->qkv + 2048, nullptr};
    a.seg[3] = {wv, m->x, m->qkv + 3072, nullptr};
    a.nseg = 4;
    a.seg_rows = 1024;
    a.K = 1024;
    a.norm_g = (const uint16_t*)m->w.attn_norm + l * kDim;
    a.seq = m->st;
    a.err = m->err;
    if (l == 0) {
      a.tokens = m->tokens;
      a.S = m->S;
      a.embd = (const uint16_t*)m->w.token_embd;
      a.embed_out = m->x;
    }
    a.trace = probe_trace(probe, Q3_KIND_QKV);
    set_prefetch(a, 0, (const uint8_t*)m->w.q8_attn_output + l * kBplO, kBplO);
    int rc = launch_q8<kOrderMlir, kModeNormIn>(a, st, launches, true);
    if (rc) return rc;
    Q3_PROBE(Q3_KIND_QKV);
    // 2) QK-norm + RoPE + KV write + attention
    AttnArgs t;
    memset(&t, 0, sizeof(t));
    t.qkv = m->qkv;
    t.q_norm = (const uint16_t*)m->w.attn_q_norm + l * kHD;
    t.k_norm = (const uint16_t*)m->w.attn_k_norm + l * kHD;
    t.rope_cos = m->rope_cos;
    t.rope_sin = m->rope_sin;
    t.rope_pos = m->S;
    t.kc = m->kc;
    t.vc = m->vc;
    t.slot0 = (int64_t)l * m->S;
    t.S = m->S;
    t.pos = &m->st->pos;
    t.pos_stride = 1;
    t.stop = stop;
    t.out = m->attn;
    t.max_chunks = max_chunks_for(m->S);
    t.part = m->att_part;
    t.counters = m->att_counters;
    t.err = m->err;
    t.trace = probe_trace(probe, Q3_KIND_ATTN);
    rc = launch_attn(t, 1, st, launches, true);
    if (rc) return rc;
    Q3_PROBE(Q3_KIND_ATTN);
    // 3) O projection + residual: h1 = x + W_o . attn
    a = q8_args_single((const uint8_t*)m->w.q8_attn_output + l * kBplO, m->attn, m->h1, m->x,
                       1024, 2048);
    a.seq = m->st;
    a.err = m->err;
    a.trace = probe_trace(probe, Q3_KIND_O);
    set_prefetch(a, 0, (const uint8_t*)m->w.q8_ffn_gate_up + l * kBplGU, kBplGU);
    rc = launch_q8<kOrderMlir, kModeResid>(a, st, launches, true);
    if (rc) return rc;
    Q3_PROBE(Q3_KIND_O);
    // 4) RMSNorm + gate|up + SwiGLU: act = swiglu(W_gu . rmsnorm(h1))
    a = q8_args_single((const uint8_t*)m->w.q8_ffn_gate_up + l * kBplGU, m->h1, m->act, nullptr,
                       3072, 1024);
    a.norm_g = (const uint16_t*)m->w.ffn_norm + l * kDim;
    a.up_off_bytes = 3072 * rb;
    a.seq = m->st;
    a.err = m->err;
    a.trace = probe_trace(probe, Q3_KIND_GATE_UP);
    set_prefetch(a, 0, (const uint8_t*)m->w.q8_ffn_down + l * kBplD, kBplD);
    rc = launch_q8<kOrderMlir, kModeSwiglu>(a, st, launches, true);
    if (rc) return rc;
    Q3_PROBE(Q3_KIND_GATE_UP);
    // 5) down projection + residual: x = h1 + W_d . act
    a = q8_args_single((const uint8_t*)m->w.q8_ffn_down + l * kBplD, m->act, m->x, m->h1, 1024,
                       3072);
    a.seq = m->st;
    a.err = m->err;
    if (ingest && l == kLayers - 1) a.advance = m->st;
    a.trace = probe_trace(probe, Q3_KIND_DOWN);
    if (l + 1 < kLayers) {
      set_prefetch(a, 0, (const uint8_t*)m->w.q8_attn_q + (l + 1) * kBplQ, kBplQ);
      set_prefetch(a, 1, (const uint8_t*)m->w.q8_attn_k + (l + 1) * kBplKV, kBplKV);
      set_prefetch(a, 2, (const uint8_t*)m->w.q8_attn_v + (l + 1) * kBplKV, kBplKV);
    }
    rc = launch_q8<kOrderMlir, kModeResid>(a, st, launches, true);
    if (rc) return rc;
    Q3_PROBE(Q3_KIND_DOWN);
  }
  return Q3_OK;
}

// The fused engine: per layer k_fused_attn then k_fused_ffn (q3_fused.cuh),
// each a grid of 8 clusters of 16 CTAs with programmatic dependent launch.
static int enqueue_layers_fused(q3_model* m, bool ingest, int* launches, const StepProbe* probe) {
  cudaStream_t st = m->stream;
  for (int l = 0; l < kLayers; ++l) {
    FaArgs fa;
    memset(&fa, 0, sizeof(fa));
    fa.wq = (const uint8_t*)m->w.q8_attn_q + l * kBplQ;
    fa.wk = (const uint8_t*)m->w.q8_attn_k + l * kBplKV;
    fa.wv = (const uint8_t*)m->w.q8_attn_v + l * kBplKV;
    fa.wo_map = m->fmaps->wo;
    fa.k_map = m->fmaps->k;
    fa.v_map = m->fmaps->v;
    fa.layer = l;
    fa.attn_norm = (const uint16_t*)m->w.attn_norm + l * kDim;
    fa.q_norm = (const uint16_t*)m->w.attn_q_norm + l * kHD;
    fa.k_norm = (const uint16_t*)m->w.attn_k_norm + l * kHD;
    if (l == 0) {
      fa.tokens = m->tokens;
      fa.embd = (const uint16_t*)m->w.token_embd;
    } else {
      fa.h1 = m->h1;
      fa.dpart = m->dpart;
    }
    fa.x_out = m->x;
    fa.opart = m->opart;
    fa.kc = m->kc;
    fa.vc = m->vc;
    fa.rope_cos = m->rope_cos;
    fa.rope_sin = m->rope_sin;
    fa.slot0 = (int64_t)l * m->S;
    fa.S = m->S;
    fa.pos = &m->st->pos;
    fa.stop = &m->st->stop;
    fa.err = m->err;
    fa.trace = probe_trace(probe, Q3_KIND_FUSED_ATTN);
    fa.phase = probe_phase(probe);
    Q3_CUDA(launch_cluster_x(k_fused_attn, dim3(kFParts * kFC), dim3(kFaThreads), kFaSmem, st,
                             true, kFC, fa));
    ++*launches;
    Q3_PROBE(Q3_KIND_FUSED_ATTN);
    FbArgs fb;
    memset(&fb, 0, sizeof(fb));
    fb.wgu = (const uint8_t*)m->w.q8_ffn_gate_up + l * kBplGU;
    fb.wd_map = m->fmaps->wd;
    fb.layer = l;
    fb.ffn_norm = (const uint16_t*)m->w.ffn_norm + l * kDim;
    fb.x = m->x;
    fb.opart = m->opart;
    fb.h1_out = m->h1;
    fb.dpart = m->dpart;
    fb.stop = &m->st->stop;
    if (ingest && l == kLayers - 1) fb.advance = m->st;
    fb.err = m->err;
    fb.trace = probe_trace(probe, Q3_KIND_FUSED_FFN);
    fb.phase = probe_phase(probe);
    Q3_CUDA(launch_cluster_x(k_fused_ffn, dim3(kFParts * kFC), dim3(kFbThreads), kFbSmem, st,
                             true, kFC, fb));
    ++*launches;
    Q3_PROBE(Q3_KIND_FUSED_FFN);
  }
  return Q3_OK;
}

static int enqueue_vocab(q3_model* m, int* launches, const StepProbe* probe, int engine) {
  cudaStream_t st = m->stream;
  VocabArgs v;
  memset(&v, 0, sizeof(v));
  v.w = (const uint16_t*)m->w.output_T;
  v.x = m->x;
  if (engine == Q3_ENGINE_FUSED) {  // x = f16(h1 + f16(sum of the last layer's down partials))
    v.xres = m->h1;
    v.xpart = m->dpart;
  }
  v.norm_g = (const uint16_t*)m->w.output_norm;
  v.logits = m->logits;
  v.N = kVocab;
  v.K = kDim;
  v.partial = m->am_part;
  v.counter = m->am_counter;
  v.seq = m->st;
  v.tokens = m->tokens;
  v.S = m->S;
  v.err = m->err;
  v.trace = probe_trace(probe, Q3_KIND_VOCAB);
  int rc = launch_vocab(v, st, launches, true);
  if (rc) return rc;
  Q3_PROBE(Q3_KIND_VOCAB);
  return Q3_OK;
}

static int capture(q3_model* m, bool ingest, cudaGraphExec_t* out, int* launches,
                   const StepProbe* probe = nullptr, int engine = Q3_ENGINE_GRAPH) {
  cudaGraph_t g = nullptr;
  Q3_CUDA(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  int n = 0;
  int rc = probe_mark(probe, m->stream, -1);
  if (rc == Q3_OK)
    rc = engine == Q3_ENGINE_FUSED ? enqueue_layers_fused(m, ingest, &n, probe)
                                   : enqueue_layers(m, ingest, &n, probe);
  if (rc == Q3_OK && !ingest) rc = enqueue_vocab(m, &n, probe, engine);
  cudaError_t e = cudaStreamEndCapture(m->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  Q3_CUDA(e);
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  Q3_CUDA(e);
  *launches = n;
  return Q3_OK;
}

static void model_free(q3_model* m) {
  if (!m) return;
  if (m->pf) prefill_destroy(m->pf);
  if (m->g_ingest) cudaGraphExecDestroy(m->g_ingest);
  if (m->g_gen) cudaGraphExecDestroy(m->g_gen);
  if (m->g_prof) cudaGraphExecDestroy(m->g_prof);
  if (m->g_ktrace) cudaGraphExecDestroy(m->g_ktrace);
  if (m->g_ingest_f) cudaGraphExecDestroy(m->g_ingest_f);
  if (m->g_gen_f) cudaGraphExecDestroy(m->g_gen_f);
  if (m->ktrace_dev) cudaFree(m->ktrace_dev);
  for (cudaEvent_t e : m->prof_events) cudaEventDestroy(e);
  void* dev[] = {m->kc, m->vc, m->rope_cos, m->rope_sin, m->x, m->qkv, m->attn, m->h1, m->act,
                 m->logits, m->tokens, m->st, m->am_part, m->att_part, m->err, m->grid_ctr,
                 m->trace_dev, m->opart, m->dpart};
  for (void* p : dev)
    if (p) cudaFree(p);
  delete m->fmaps;
  if (m->h_st) cudaFreeHost(m->h_st);
  if (m->h_tokens) cudaFreeHost(m->h_tokens);
  if (m->own_stream && m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

#define Q3_MALLOC(ptr, bytes)                                                        \
  do {                                                                               \
    cudaError_t e_ = cudaMalloc((void**)&(ptr), (bytes));                            \
    if (e_ != cudaSuccess) {                                                         \
      cudaGetLastError();                                                            \
      model_free(m);                                                                 \
      return set_err(Q3_ERR_NOMEM, "cudaMalloc(%zu) for %s failed: %s", (size_t)(bytes), \
                     #ptr, cudaGetErrorString(e_));                                  \
    }                                                                                \
  } while (0)

// The persistent engine needs one co-resident CTA per SM (cooperative launch).
static int persist_setup(q3_model* m) {
  Q3_CUDA(cudaFuncSetAttribute(k_decode_persistent, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)kPersistSmem));
  int per_sm = 0;
  Q3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_persistent,
                                                          kGemvThreads, kPersistSmem));
  int coop = 0;
  Q3_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device));
  m->persist_grid = (per_sm >= 1 && coop) ? current_sms() : 0;
  if (m->persist_grid > kArgmaxMaxGrid) m->persist_grid = 0;
  Q3_CUDA(cudaMalloc((void**)&m->grid_ctr, 256));
  Q3_CUDA(cudaMemset(m->grid_ctr, 0, 256));
  return Q3_OK;
}

// The fused engine needs caches of at most kFusedMaxPositions positions and
// 16-CTA clusters of both of its kernels resident (non-portable size).
static int fused_setup(q3_model* m) {
  m->fused_clusters = 0;
  if (m->S > kFusedMaxPositions) return Q3_OK;
  int rc = fused_attrs();
  if (rc) return rc;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kFC;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kFParts * kFC);
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int na = 0, nb = 0;
  cfg.blockDim = dim3(kFaThreads);
  cfg.dynamicSmemBytes = kFaSmem;
  if (cudaOccupancyMaxActiveClusters(&na, (void*)k_fused_attn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    na = 0;
  }
  cfg.blockDim = dim3(kFbThreads);
  cfg.dynamicSmemBytes = kFbSmem;
  if (cudaOccupancyMaxActiveClusters(&nb, (void*)k_fused_ffn, &cfg) != cudaSuccess) {
    cudaGetLastError();
    nb = 0;
  }
  m->fused_clusters = na < nb ? na : nb;
  if (m->fused_clusters < 1) return Q3_OK;
  m->fmaps = new FusedMaps();
  rc = make_fused_maps(m->fmaps, &m->w, m->kc, m->vc, (int64_t)kLayers * m->S);
  if (rc) {
    m->fused_clusters = 0;
    return rc;
  }
  Q3_CUDA(cudaMalloc((void**)&m->opart, kFParts * kDim * sizeof(float)));
  Q3_CUDA(cudaMalloc((void**)&m->dpart, kFParts * kDim * sizeof(float)));
  Q3_CUDA(cudaMemset(m->opart, 0, kFParts * kDim * sizeof(float)));
  Q3_CUDA(cudaMemset(m->dpart, 0, kFParts * kDim * sizeof(float)));
  return Q3_OK;
}

extern "C" int q3_model_create(const q3_weights* w, int64_t S, void* stream, q3_model** out) {
  Q3_REQUIRE(w && out, "null pointer");
  Q3_REQUIRE(S >= 2 && S <= (1 << 20), "max_seq_len=%lld out of range", (long long)S);
  const void* req[] = {w->token_embd, w->output_norm, w->output_T, w->attn_norm, w->ffn_norm,
                       w->attn_q_norm, w->attn_k_norm, w->q8_attn_q, w->q8_attn_k, w->q8_attn_v,
                       w->q8_attn_output, w->q8_ffn_gate_up, w->q8_ffn_down};
  for (const void* p : req) {
    Q3_REQUIRE(p != nullptr, "a weight pointer is null");
    Q3_REQUIRE(aligned16(p), "weight pointers must be 16-byte aligned");
  }
  int dev = 0;
  Q3_CUDA(cudaGetDevice(&dev));
  int major = 0;
  Q3_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  if (major != 10) return set_err(Q3_ERR_UNSUPPORTED, "device %d is sm_%d0; this build is sm_100a", dev, major);
  q3_model* m = new q3_model();
  m->device = dev;
  m->w = *w;
  m->S = S;
  if (stream) {
    m->stream = (cudaStream_t)stream;
  } else {
    cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      model_free(m);
      return set_err(Q3_ERR_CUDA, "stream create: %s", cudaGetErrorString(e));
    }
    m->own_stream = true;
  }
  const size_t cache = (size_t)kLayers * S * kNKV * kHD * sizeof(uint16_t);
  Q3_MALLOC(m->kc, cache);
  Q3_MALLOC(m->vc, cache);
  Q3_MALLOC(m->rope_cos, (size_t)S * 64 * sizeof(float));
  Q3_MALLOC(m->rope_sin, (size_t)S * 64 * sizeof(float));
  Q3_MALLOC(m->x, kDim * 2);
  Q3_MALLOC(m->qkv, 4096 * 2);
  Q3_MALLOC(m->attn, 2048 * 2);
  Q3_MALLOC(m->h1, kDim * 2);
  Q3_MALLOC(m->act, kFFN * 2);
  Q3_MALLOC(m->logits, (size_t)kVocab * 2);
  Q3_MALLOC(m->tokens, (size_t)(S + 1) * sizeof(int64_t));
  Q3_MALLOC(m->st, sizeof(SeqState));
  Q3_MALLOC(m->am_part, q3_vocab_argmax_workspace_bytes());
  m->am_counter = (unsigned int*)((uint8_t*)m->am_part + sizeof(ArgmaxPartial) * kArgmaxMaxGrid);
  Q3_MALLOC(m->att_part, q3_attention_workspace_bytes(S));
  m->att_counters = (unsigned int*)((uint8_t*)m->att_part +
                                    sizeof(AttnPartial) * (size_t)kNKV * max_chunks_for(S) * 2);
  Q3_MALLOC(m->err, sizeof(int));
  if (cudaMallocHost((void**)&m->h_st, sizeof(SeqState)) != cudaSuccess ||
      cudaMallocHost((void**)&m->h_tokens, (size_t)(S + 1) * sizeof(int64_t)) != cudaSuccess) {
    cudaGetLastError();
    model_free(m);
    return set_err(Q3_ERR_NOMEM, "pinned host allocation failed");
  }
  std::vector<float> c((size_t)S * 64), s((size_t)S * 64);
  q3_rope_table(S, c.data(), s.data());
  int rc = Q3_OK;
  auto chk = [&](cudaError_t e) {
    if (e != cudaSuccess && rc == Q3_OK)
      rc = set_err(Q3_ERR_CUDA, "model init: %s", cudaGetErrorString(e));
  };
  chk(cudaMemcpyAsync(m->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice, m->stream));
  chk(cudaMemcpyAsync(m->rope_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice, m->stream));
  chk(cudaMemsetAsync(m->am_part, 0, q3_vocab_argmax_workspace_bytes(), m->stream));
  chk(cudaMemsetAsync(m->att_part, 0, q3_attention_workspace_bytes(S), m->stream));
  chk(cudaMemsetAsync(m->err, 0, sizeof(int), m->stream));
  chk(cudaMemsetAsync(m->st, 0, sizeof(SeqState), m->stream));
  chk(cudaMemsetAsync(m->tokens, 0, (size_t)(S + 1) * sizeof(int64_t), m->stream));
  chk(cudaStreamSynchronize(m->stream));
  if (rc == Q3_OK) rc = capture(m, true, &m->g_ingest, &m->launches_ingest);
  if (rc == Q3_OK) rc = capture(m, false, &m->g_gen, &m->launches_gen);
  if (rc == Q3_OK) rc = persist_setup(m);
  if (rc == Q3_OK) rc = fused_setup(m);
  if (rc == Q3_OK && m->fused_clusters > 0)
    rc = capture(m, true, &m->g_ingest_f, &m->launches_ingest_f, nullptr, Q3_ENGINE_FUSED);
  if (rc == Q3_OK && m->fused_clusters > 0)
    rc = capture(m, false, &m->g_gen_f, &m->launches_gen_f, nullptr, Q3_ENGINE_FUSED);
  if (rc != Q3_OK) {
    model_free(m);
    return rc;
  }
  // default: the fused engine where it is available
  m->engine = m->fused_clusters > 0 ? Q3_ENGINE_FUSED : Q3_ENGINE_GRAPH;
  const char* env = getenv("Q3_ENGINE");
  if (env && strcmp(env, "graph") == 0) m->engine = Q3_ENGINE_GRAPH;
  if (env && strcmp(env, "fused") == 0 && m->fused_clusters > 0) m->engine = Q3_ENGINE_FUSED;
  if (env && strcmp(env, "persistent") == 0 && m->persist_grid > 0) m->engine = Q3_ENGINE_PERSISTENT;
  *out = m;
  return Q3_OK;
}

extern "C" int q3_model_set_prefill(q3_model* m, int mode) {
  Q3_REQUIRE(m, "null model");
  Q3_REQUIRE(mode == Q3_PREFILL_STEPS || mode == Q3_PREFILL_BATCHED, "unknown prefill mode %d", mode);
  m->prefill_mode = mode;
  return Q3_OK;
}

extern "C" int q3_model_prefill_mode(q3_model* m, int* mode) {
  Q3_REQUIRE(m && mode, "null pointer");
  *mode = m->prefill_mode;
  return Q3_OK;
}

extern "C" int q3_model_set_engine(q3_model* m, int engine) {
  Q3_REQUIRE(m, "null model");
  Q3_REQUIRE(engine == Q3_ENGINE_GRAPH || engine == Q3_ENGINE_PERSISTENT ||
                 engine == Q3_ENGINE_FUSED,
             "unknown engine %d", engine);
  if (engine == Q3_ENGINE_PERSISTENT && m->persist_grid == 0)
    return set_err(Q3_ERR_UNSUPPORTED, "the persistent kernel cannot be co-resident here");
  if (engine == Q3_ENGINE_FUSED && m->fused_clusters == 0)
    return set_err(Q3_ERR_UNSUPPORTED,
                   "the fused engine needs max_seq_len <= %lld and resident 16-CTA clusters",
                   (long long)kFusedMaxPositions);
  m->engine = engine;
  return Q3_OK;
}

extern "C" int q3_model_engine(q3_model* m, int* engine) {
  Q3_REQUIRE(m && engine, "null pointer");
  *engine = m->engine;
  return Q3_OK;
}

extern "C" int q3_model_kernel_launches(q3_model* m, int64_t* n) {
  Q3_REQUIRE(m && n, "null pointer");
  *n = m->kernel_launches;
  return Q3_OK;
}

extern "C" int q3_model_destroy(q3_model* m) {
  if (m) {
    cudaStreamSynchronize(m->stream);
    model_free(m);
  }
  return Q3_OK;
}

extern "C" void* q3_model_stream(q3_model* m) { return m ? (void*)m->stream : nullptr; }

extern "C" int q3_model_launches_per_step(q3_model* m, int64_t* n) {
  Q3_REQUIRE(m && n, "null pointer");
  *n = m->engine == Q3_ENGINE_FUSED ? m->launches_gen_f : m->engine == Q3_ENGINE_PERSISTENT ? 1
                                                                                          : m->launches_gen;
  return Q3_OK;
}

extern "C" int q3_model_poke(q3_model* m, int what, int64_t index, int64_t value) {
  Q3_REQUIRE(m, "null model");
  if (what == Q3_POKE_TOKEN) {
    Q3_REQUIRE(index >= 0 && index <= m->S, "token index %lld outside [0, %lld]",
               (long long)index, (long long)m->S);
    Q3_CUDA(cudaMemcpyAsync(m->tokens + index, &value, sizeof(int64_t), cudaMemcpyHostToDevice,
                            m->stream));
  } else if (what == Q3_POKE_POS) {
    Q3_CUDA(cudaMemcpyAsync(&m->st->pos, &value, sizeof(int64_t), cudaMemcpyHostToDevice,
                            m->stream));
  } else {
    return set_err(Q3_ERR_INVALID, "unknown poke %d", what);
  }
  Q3_CUDA(cudaStreamSynchronize(m->stream));
  return Q3_OK;
}

extern "C" int q3_model_device_error(q3_model* m, int* code) {
  Q3_REQUIRE(m && code, "null pointer");
  Q3_CUDA(cudaMemcpyAsync(code, m->err, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
  Q3_CUDA(cudaStreamSynchronize(m->stream));
  return Q3_OK;
}

// Upload tokens at positions [pos0, pos0+n) and a fresh sequence state.
// Tokens toks[0..n) at positions pos0.. and the step state; the first step
// feeds position state_pos (pos0, or where a prefill stopped).
static int seq_begin(q3_model* m, const int64_t* toks, int64_t pos0, int64_t n, int64_t n_prompt,
                     int64_t max_gen, int64_t eos, int64_t state_pos = -1) {
  memcpy(m->h_tokens, toks, (size_t)n * sizeof(int64_t));
  Q3_CUDA(cudaMemcpyAsync(m->tokens + pos0, m->h_tokens, (size_t)n * sizeof(int64_t),
                          cudaMemcpyHostToDevice, m->stream));
  SeqState s;
  memset(&s, 0, sizeof(s));
  s.pos = state_pos >= 0 ? state_pos : pos0;
  s.n_prompt = n_prompt;
  s.max_gen = max_gen;
  s.eos = eos;
  s.stop = 0;
  *m->h_st = s;
  Q3_CUDA(cudaMemcpyAsync(m->st, m->h_st, sizeof(SeqState), cudaMemcpyHostToDevice, m->stream));
  Q3_CUDA(cudaMemsetAsync(m->err, 0, sizeof(int), m->stream));
  return Q3_OK;
}

// Enqueue n_ingest prompt steps (no vocab head) then n_gen steps that end
// with the vocab head + argmax, on the model's engine.
static int launch_graphs(q3_model* m, int64_t n_ingest, int64_t n_gen) {
  if (n_ingest + n_gen == 0) return Q3_OK;
  if (m->engine == Q3_ENGINE_PERSISTENT) {
    PersistArgs a;
    memset(&a, 0, sizeof(a));
    a.token_embd = (const uint16_t*)m->w.token_embd;
    a.output_norm = (const uint16_t*)m->w.output_norm;
    a.output_T = (const uint16_t*)m->w.output_T;
    a.attn_norm = (const uint16_t*)m->w.attn_norm;
    a.ffn_norm = (const uint16_t*)m->w.ffn_norm;
    a.q_norm = (const uint16_t*)m->w.attn_q_norm;
    a.k_norm = (const uint16_t*)m->w.attn_k_norm;
    a.wq = (const uint8_t*)m->w.q8_attn_q;
    a.wk = (const uint8_t*)m->w.q8_attn_k;
    a.wv = (const uint8_t*)m->w.q8_attn_v;
    a.wo = (const uint8_t*)m->w.q8_attn_output;
    a.wgu = (const uint8_t*)m->w.q8_ffn_gate_up;
    a.wd = (const uint8_t*)m->w.q8_ffn_down;
    a.kc = m->kc;
    a.vc = m->vc;
    a.rope_cos = m->rope_cos;
    a.rope_sin = m->rope_sin;
    a.S = m->S;
    a.x = m->x;
    a.qkv = m->qkv;
    a.attn = m->attn;
    a.h1 = m->h1;
    a.act = m->act;
    a.logits = m->logits;
    a.tokens = m->tokens;
    a.seq = m->st;
    a.am_part = m->am_part;
    a.am_counter = m->am_counter;
    a.att_part = m->att_part;
    a.att_counters = m->att_counters;
    a.max_chunks = max_chunks_for(m->S);
    a.grid_ctr = m->grid_ctr;
    a.err = m->err;
    a.n_steps = (int)(n_ingest + n_gen);
    a.vocab_from = (int)n_ingest;
    a.trace = m->trace_dev;
    a.trace_step = m->trace_step;
    // counters start at zero (they re-arm themselves, unless a run was cut short)
    Q3_CUDA(cudaMemsetAsync(m->grid_ctr, 0, sizeof(unsigned int), m->stream));
    Q3_CUDA(cudaMemsetAsync(m->am_counter, 0, sizeof(unsigned int), m->stream));
    Q3_CUDA(cudaMemsetAsync(m->att_counters, 0, kNKV * sizeof(unsigned int), m->stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->persist_grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = kPersistSmem;
    cfg.stream = m->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q3_CUDA(cudaLaunchKernelEx(&cfg, k_decode_persistent, a));
    m->kernel_launches += 1;
    return Q3_OK;
  }
  const bool f = m->engine == Q3_ENGINE_FUSED;
  cudaGraphExec_t gi = f ? m->g_ingest_f : m->g_ingest, gg = f ? m->g_gen_f : m->g_gen;
  for (int64_t i = 0; i < n_ingest; ++i) Q3_CUDA(cudaGraphLaunch(gi, m->stream));
  for (int64_t i = 0; i < n_gen; ++i) Q3_CUDA(cudaGraphLaunch(gg, m->stream));
  m->kernel_launches += n_ingest * (f ? m->launches_ingest_f : m->launches_ingest) +
                        n_gen * (f ? m->launches_gen_f : m->launches_gen);
  return Q3_OK;
}

static int check_device_err(q3_model* m) {
  int code = 0;
  Q3_CUDA(cudaMemcpyAsync(&code, m->err, sizeof(int), cudaMemcpyDeviceToHost, m->stream));
  Q3_CUDA(cudaStreamSynchronize(m->stream));
  if (code != 0) return set_err(Q3_ERR_DEVICE, "kernel error word %d", code);
  return Q3_OK;
}

extern "C" int q3_generate_begin(q3_model* m, const int64_t* prompt, int64_t n_prompt,
                                 int64_t max_gen, int64_t eos) {
  Q3_REQUIRE(m && prompt, "null pointer");
  Q3_REQUIRE(n_prompt >= 1, "the prompt must hold at least one token");
  Q3_REQUIRE(max_gen >= 0, "max_gen must be >= 0");
  Q3_REQUIRE(n_prompt + max_gen <= m->S, "n_prompt + max_gen = %lld exceeds max_seq_len %lld",
             (long long)(n_prompt + max_gen), (long long)m->S);
  for (int64_t i = 0; i < n_prompt; ++i)
    Q3_REQUIRE(prompt[i] >= 0 && prompt[i] < kVocab, "prompt token %lld out of range",
               (long long)prompt[i]);
  // all but the last prompt token are ingested (no vocab head); the last one
  // runs the vocab head.  Batched prefill writes the ingested positions' K/V
  // rows in passes of up to 64 positions instead of one decode step each.
  const bool pf = m->prefill_mode == Q3_PREFILL_BATCHED && n_prompt > 1;
  int rc = seq_begin(m, prompt, 0, n_prompt, n_prompt, max_gen, eos, pf ? n_prompt - 1 : 0);
  if (rc) return rc;
  m->gen_n_prompt = n_prompt;
  m->gen_pos0 = 0;
  m->gen_max = max_gen;
  m->gen_active = true;
  if (pf) {
    if ((rc = model_prefill(m, 0, n_prompt - 1))) return rc;
    return launch_graphs(m, 0, 1);
  }
  return launch_graphs(m, n_prompt - 1, 1);
}

extern "C" int q3_generate_steps(q3_model* m, int64_t steps) {
  Q3_REQUIRE(m, "null model");
  if (!m->gen_active) return set_err(Q3_ERR_STATE, "no generation in progress");
  return launch_graphs(m, 0, steps);
}

static int read_generated(q3_model* m, int64_t first_pos, int64_t max_gen, int64_t* out,
                          int64_t* n_out) {
  if (max_gen > 0)
    Q3_CUDA(cudaMemcpyAsync(m->h_tokens, m->tokens + first_pos, (size_t)max_gen * sizeof(int64_t),
                            cudaMemcpyDeviceToHost, m->stream));
  Q3_CUDA(cudaMemcpyAsync(m->h_st, m->st, sizeof(SeqState), cudaMemcpyDeviceToHost, m->stream));
  int rc = check_device_err(m);
  if (rc) return rc;
  const int64_t n = m->h_st->n_gen;
  if (out && n > 0) memcpy(out, m->h_tokens, (size_t)n * sizeof(int64_t));
  if (n_out) *n_out = n;
  return Q3_OK;
}

extern "C" int q3_generate_end(q3_model* m, int64_t* out, int64_t* n_out) {
  Q3_REQUIRE(m, "null model");
  if (!m->gen_active) return set_err(Q3_ERR_STATE, "no generation in progress");
  m->gen_active = false;
  // generated tokens sit at positions n_prompt+1 .. (the first token, at n_prompt, is fed only)
  return read_generated(m, m->gen_pos0 + m->gen_n_prompt + 1, m->gen_max, out, n_out);
}

extern "C" int q3_run(q3_model* m, const int64_t* prompt, int64_t n_prompt, int64_t max_gen,
                      int64_t eos, int64_t* out, int64_t* n_out) {
  Q3_REQUIRE(out || max_gen == 0, "out_tokens is null");
  int rc = q3_generate_begin(m, prompt, n_prompt, max_gen, eos);
  if (rc) return rc;
  rc = q3_generate_steps(m, max_gen);
  if (rc) return rc;
  return q3_generate_end(m, out, n_out);
}

extern "C" int q3_decode(q3_model* m, int64_t token, int64_t pos, void* logits, int64_t* next) {
  Q3_REQUIRE(m, "null model");
  Q3_REQUIRE(token >= 0 && token < kVocab, "token out of range");
  Q3_REQUIRE(pos >= 0 && pos < m->S, "pos out of range");
  m->gen_active = false;
  int rc = seq_begin(m, &token, pos, 1, INT64_MAX / 2, INT64_MAX / 2, -1);
  if (rc) return rc;
  rc = launch_graphs(m, 0, 1);
  if (rc) return rc;
  if (logits)
    Q3_CUDA(cudaMemcpyAsync(logits, m->logits, (size_t)kVocab * 2, cudaMemcpyDeviceToDevice,
                            m->stream));
  Q3_CUDA(cudaMemcpyAsync(m->h_tokens, m->tokens + pos + 1, sizeof(int64_t),
                          cudaMemcpyDeviceToHost, m->stream));
  rc = check_device_err(m);
  if (rc) return rc;
  if (next) *next = m->h_tokens[0];
  return Q3_OK;
}

extern "C" int q3_init_chat(q3_model* m, int64_t max_ctx) {
  Q3_REQUIRE(m, "null model");
  Q3_REQUIRE(max_ctx >= 2 && max_ctx <= m->S, "max_ctx must be in [2, max_seq_len]");
  const size_t cache = (size_t)kLayers * m->S * kNKV * kHD * sizeof(uint16_t);
  Q3_CUDA(cudaMemsetAsync(m->kc, 0, cache, m->stream));
  Q3_CUDA(cudaMemsetAsync(m->vc, 0, cache, m->stream));
  Q3_CUDA(cudaStreamSynchronize(m->stream));
  m->chat_ready = true;
  m->chat_pos = 0;
  m->chat_max = max_ctx;
  m->gen_active = false;
  return Q3_OK;
}

extern "C" int q3_chat_turn(q3_model* m, const int64_t* toks, int64_t n, int64_t max_gen,
                            int64_t eos, int64_t* out, int64_t* n_out) {
  Q3_REQUIRE(m && toks, "null pointer");
  if (!m->chat_ready) return set_err(Q3_ERR_STATE, "q3_init_chat was not called");
  Q3_REQUIRE(n >= 1 && max_gen >= 0, "need n_tokens >= 1 and max_gen >= 0");
  Q3_REQUIRE(m->chat_pos + n + max_gen <= m->chat_max, "turn exceeds the chat context");
  Q3_REQUIRE(out || max_gen == 0, "out_tokens is null");
  for (int64_t i = 0; i < n; ++i)
    Q3_REQUIRE(toks[i] >= 0 && toks[i] < kVocab, "token out of range");
  const int64_t p0 = m->chat_pos;
  const bool pf = m->prefill_mode == Q3_PREFILL_BATCHED && n > 1;
  int rc = seq_begin(m, toks, p0, n, p0 + n, max_gen, eos, pf ? p0 + n - 1 : p0);
  if (rc) return rc;
  if (pf && (rc = model_prefill(m, p0, n - 1))) return rc;
  rc = launch_graphs(m, pf ? 0 : n - 1, 1 + max_gen);
  if (rc) return rc;
  int64_t got = 0;
  rc = read_generated(m, p0 + n + 1, max_gen, out, &got);
  if (rc) return rc;
  if (n_out) *n_out = got;
  // model/qwen3_full.mlir:2216-2218: current_pos = new_pos + (count + 1)
  m->chat_pos = p0 + n + got + 1;
  return Q3_OK;
}

extern "C" int q3_model_profile_steps(q3_model* m, int64_t steps, float* times_us, int32_t* kinds,
                                      int64_t cap) {
  Q3_REQUIRE(m && times_us && kinds && steps >= 1, "bad arguments");
  if (!m->gen_active) return set_err(Q3_ERR_STATE, "no generation in progress");
  const int eng = m->engine == Q3_ENGINE_FUSED ? Q3_ENGINE_FUSED : Q3_ENGINE_GRAPH;
  if (m->g_prof && m->prof_engine != eng) {
    cudaGraphExecDestroy(m->g_prof);
    m->g_prof = nullptr;
    for (cudaEvent_t e : m->prof_events) cudaEventDestroy(e);
    m->prof_events.clear();
    m->prof_kinds.clear();
  }
  if (!m->g_prof) {
    StepProbe pr{&m->prof_events, &m->prof_kinds};
    int n = 0;
    int rc = capture(m, false, &m->g_prof, &n, &pr, eng);
    if (rc) return rc;
    m->prof_engine = eng;
  }
  const int64_t nk = (int64_t)m->prof_events.size() - 1;
  Q3_REQUIRE(cap >= nk, "cap %lld below the %lld kernels of a step", (long long)cap, (long long)nk);
  std::vector<double> acc((size_t)nk, 0.0);
  for (int64_t s = 0; s < steps; ++s) {
    Q3_CUDA(cudaGraphLaunch(m->g_prof, m->stream));
    Q3_CUDA(cudaStreamSynchronize(m->stream));
    for (int64_t i = 0; i < nk; ++i) {
      float ms = 0.0f;
      Q3_CUDA(cudaEventElapsedTime(&ms, m->prof_events[i], m->prof_events[i + 1]));
      acc[(size_t)i] += ms;
    }
  }
  for (int64_t i = 0; i < nk; ++i) {
    times_us[i] = (float)(acc[(size_t)i] / (double)steps * 1000.0);
    kinds[i] = m->prof_kinds[(size_t)i + 1];
  }
  return Q3_OK;
}

// Timing of every kernel of `steps` graph-engine decode steps (which advance
// the sequence): out[k][0..5] = first CTA start, first and last release from
// the wait on the previous kernel, last CTA end, last CTA start, first CTA
// end, in ns from the step's first kernel start, averaged over the steps;
// kinds[k] = Q3_KIND_*.
extern "C" int q3_model_trace_kernels(q3_model* m, int64_t steps, long long* out, int32_t* kinds,
                                      int64_t cap, int64_t* n_kernels) {
  Q3_REQUIRE(m && out && kinds && n_kernels && steps >= 1, "bad arguments");
  if (!m->gen_active) return set_err(Q3_ERR_STATE, "no generation in progress");
  constexpr int kMaxTraced = 512;
  const int eng = m->engine == Q3_ENGINE_FUSED ? Q3_ENGINE_FUSED : Q3_ENGINE_GRAPH;
  if (m->g_ktrace && m->ktrace_engine != eng) {
    cudaGraphExecDestroy(m->g_ktrace);
    m->g_ktrace = nullptr;
  }
  if (!m->g_ktrace) {
    if (!m->ktrace_dev) Q3_CUDA(cudaMalloc((void**)&m->ktrace_dev, kMaxTraced * kTraceVals * 8));
    int slot = 0, n = 0;
    m->ktrace_kinds.clear();
    StepProbe pr;
    pr.ktrace = m->ktrace_dev;
    pr.slot = &slot;
    pr.tkinds = &m->ktrace_kinds;
    int rc = capture(m, false, &m->g_ktrace, &n, &pr, eng);
    if (rc) return rc;
    m->ktrace_engine = eng;
  }
  const int64_t nk = (int64_t)m->ktrace_kinds.size();
  *n_kernels = nk;
  Q3_REQUIRE(cap >= nk && nk <= kMaxTraced, "cap %lld below the %lld kernels of a step",
             (long long)cap, (long long)nk);
  constexpr int V = kTraceVals;
  std::vector<unsigned long long> init((size_t)nk * V, 0ull), rec((size_t)nk * V);
  for (int64_t k = 0; k < nk; ++k) init[k * V + 0] = init[k * V + 1] = init[k * V + 5] = ~0ull;
  std::vector<double> acc((size_t)nk * V, 0.0);
  for (int64_t s = 0; s < steps; ++s) {
    Q3_CUDA(cudaMemcpyAsync(m->ktrace_dev, init.data(), init.size() * 8, cudaMemcpyHostToDevice,
                            m->stream));
    Q3_CUDA(cudaGraphLaunch(m->g_ktrace, m->stream));
    Q3_CUDA(cudaMemcpyAsync(rec.data(), m->ktrace_dev, rec.size() * 8, cudaMemcpyDeviceToHost,
                            m->stream));
    Q3_CUDA(cudaStreamSynchronize(m->stream));
    unsigned long long t0 = ~0ull;
    for (int64_t k = 0; k < nk; ++k) t0 = std::min(t0, rec[k * V]);
    for (size_t i = 0; i < rec.size(); ++i)
      acc[i] += (rec[i] == ~0ull || rec[i] == 0) ? 0.0 : (double)(rec[i] - t0);
  }
  m->kernel_launches += steps * nk;
  for (int64_t k = 0; k < nk; ++k) {
    kinds[k] = m->ktrace_kinds[(size_t)k];
    for (int j = 0; j < 6; ++j) out[k * 6 + j] = (long long)(acc[k * V + j] / (double)steps);
  }
  return Q3_OK;
}

// Per-CTA phase stamps of the fused engine's kernels during the last of
// `steps` decode steps (which advance the sequence): out[launch][cta][phase]
// in ns of %globaltimer, 2 x 28 launches of 128 CTAs x kFPhases each.
extern "C" int q3_model_trace_phases(q3_model* m, int64_t steps, long long* out, int64_t cap,
                                     int64_t* n_launches, int* ctas, int* phases) {
  Q3_REQUIRE(m && out && n_launches && ctas && phases && steps >= 1, "bad arguments");
  if (!m->gen_active) return set_err(Q3_ERR_STATE, "no generation in progress");
  if (m->engine != Q3_ENGINE_FUSED) return set_err(Q3_ERR_STATE, "phase tracing needs the fused engine");
  const int64_t nl = 2 * kLayers, per = (int64_t)kFParts * kFC * kFPhases;
  Q3_REQUIRE(cap >= nl * per, "cap %lld below %lld", (long long)cap, (long long)(nl * per));
  long long* dev = nullptr;
  Q3_CUDA(cudaMalloc((void**)&dev, (size_t)(nl * per) * sizeof(long long)));
  Q3_CUDA(cudaMemset(dev, 0, (size_t)(nl * per) * sizeof(long long)));
  cudaGraphExec_t g = nullptr;
  int n = 0, ps = 0;
  StepProbe pr;
  pr.phase = dev;
  pr.pslot = &ps;
  int rc = capture(m, false, &g, &n, &pr, Q3_ENGINE_FUSED);
  for (int64_t i = 0; rc == Q3_OK && i < steps; ++i) {
    const cudaError_t e = cudaGraphLaunch(g, m->stream);
    if (e != cudaSuccess) rc = set_err(Q3_ERR_CUDA, "trace launch: %s", cudaGetErrorString(e));
  }
  if (rc == Q3_OK) {
    cudaError_t e = cudaMemcpyAsync(out, dev, (size_t)(nl * per) * sizeof(long long),
                                    cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) rc = set_err(Q3_ERR_CUDA, "trace copy: %s", cudaGetErrorString(e));
  }
  if (g) cudaGraphExecDestroy(g);
  cudaFree(dev);
  m->kernel_launches += steps * n;
  *n_launches = nl;
  *ctas = kFParts * kFC;
  *phases = kFPhases;
  return rc;
}

extern "C" int q3_model_trace_steps(q3_model* m, int64_t steps, int64_t trace_step,
                                    long long* out, int64_t cap, int* ctas, int* phases) {
  Q3_REQUIRE(m && out && ctas && phases && steps >= 1, "bad arguments");
  Q3_REQUIRE(trace_step >= 0 && trace_step < steps, "trace_step outside the launch");
  if (!m->gen_active) return set_err(Q3_ERR_STATE, "no generation in progress");
  if (m->engine != Q3_ENGINE_PERSISTENT) return set_err(Q3_ERR_STATE, "tracing needs the persistent engine");
  const int64_t n = (int64_t)m->persist_grid * kTracePhases * 4;
  Q3_REQUIRE(cap >= n, "cap %lld below %lld", (long long)cap, (long long)n);
  if (!m->trace_dev) Q3_CUDA(cudaMalloc((void**)&m->trace_dev, (size_t)n * sizeof(long long)));
  Q3_CUDA(cudaMemsetAsync(m->trace_dev, 0, (size_t)n * sizeof(long long), m->stream));
  m->trace_step = (int)trace_step;
  int rc = launch_graphs(m, 0, steps);
  m->trace_step = -1;
  long long* dev = m->trace_dev;
  m->trace_dev = nullptr;
  if (rc == Q3_OK) {
    cudaError_t e = cudaMemcpyAsync(out, dev, (size_t)n * sizeof(long long), cudaMemcpyDeviceToHost,
                                    m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) rc = set_err(Q3_ERR_CUDA, "trace copy: %s", cudaGetErrorString(e));
  }
  m->trace_dev = dev;
  *ctas = m->persist_grid;
  *phases = kTracePhases;
  return rc;
}

// ---------------------------------------------------------------------------
// batched decoder (tcgen05 projections and vocab head)
// ---------------------------------------------------------------------------
#include "q3_batch.cuh"
#include "q3_battn.cuh"
#include "q3_batch_host.inc"
