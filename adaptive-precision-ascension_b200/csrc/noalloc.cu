// Bias gradient for callers that cannot allocate device memory.
//
// apa_bias_grad_noalloc computes exactly what apa_cast (with column partial
// sums) followed by apa_colsum_finalize computes, but the partial sums live in
// a fixed array compiled into this library instead of a buffer the caller
// allocates. It is meant for callers that must not call cudaMalloc at the
// point where they need the bias gradient, for example:
//   * a host framework that owns all device memory through its own arena or
//     pool and does not let libraries allocate behind its back;
//   * code running between stream operations of another runtime, where
//     cudaMalloc/cudaFree would implicitly synchronise the device and stall
//     work that is already queued;
//   * bindings from other languages that only receive device pointers to
//     buffers owned elsewhere and have no allocator to hand out scratch.
//
// The scratch array holds kScratchFloats fp32 partial sums (16 MiB), enough for
// ceil(rows / 64) * cols <= 4 Mi, e.g. 8192 x 32768 or 65536 x 4096. Larger
// problems are rejected with APA_ERR_NOALLOC_LIMIT before anything is launched.
// Every GPU that loads the library keeps this array for the life of the
// process.
//
// The array is shared by every call on a device and keeps whatever the last
// call left in it. Each call overwrites every partial sum it later reads, so
// nothing needs clearing between calls; but two calls that run at the same
// time on the GPU (different streams, or different host threads with no
// ordering between their streams) write the same array and race. Order such
// calls on one stream.
//
// The first call on a device looks up the device address of the array (with
// that device current) and caches it; host code never passes the array's
// name to a kernel, since on the host that name is only a stand-in for the
// device symbol. Make that first call before any stream capture. The cache
// remembers the CUDA context it was taken in (the driver's context ID, unique
// for the life of the process): when the device's context has changed since
// (cudaDeviceReset, or a primary context released and created again), the
// next call looks the address up again in the new context. That call is then
// a first call again and belongs before any stream capture too.
#include <cuda.h>
#include <mutex>

#include "apa_common.cuh"

namespace apa {
namespace noalloc {

constexpr int64_t kScratchFloats = int64_t(4) << 20;   // 16 MiB of fp32 partial sums
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_bias_scratch[kScratchFloats];

std::mutex g_mutex;
float* g_device_addr[kMaxDevices] = {};
unsigned long long g_ctx_id[kMaxDevices] = {};   // context the address belongs to (0: unknown)

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// ID of the calling thread's current context, 0 when it cannot be told (no
// current context, or a driver without cuCtxGetId).
unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_bias_scratch on the current device: looked up once per
// device, and again when the device's context is not the one it was taken in.
int scratch_address(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return APA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return APA_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_mutex);
  const unsigned long long id = current_ctx_id();
  if (g_device_addr[dev] == nullptr || (id != 0 && id != g_ctx_id[dev])) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_bias_scratch) != cudaSuccess || p == nullptr) return APA_ERR_CUDA;
    g_device_addr[dev] = static_cast<float*>(p);
    g_ctx_id[dev] = current_ctx_id();   // the lookup made the device's context current
  }
  *out = g_device_addr[dev];
  return APA_OK;
}

}  // namespace noalloc
}  // namespace apa

extern "C" int apa_bias_grad_noalloc(const void* dy, int dy_dtype, int64_t rows, int64_t cols, int64_t ld,
                                     int work_dtype, float* db, int accumulate, void* stream) {
  using namespace apa;
  if (!dy || !db || rows <= 0 || cols <= 0 || ld < cols) return APA_ERR_INVALID;
  if (dy_dtype != APA_DT_F32 && dy_dtype != APA_DT_F16 && dy_dtype != APA_DT_BF16) return APA_ERR_UNSUPPORTED;
  if (work_dtype != APA_DT_E4M3 && work_dtype != APA_DT_F16 && work_dtype != APA_DT_F32) return APA_ERR_UNSUPPORTED;
  const int64_t nparts = (rows + 63) / 64;
  if (nparts > noalloc::kScratchFloats / cols) return APA_ERR_NOALLOC_LIMIT;
  float* scratch = nullptr;
  if (int st = noalloc::scratch_address(&scratch)) return st;

  CastParams p;
  p.src = dy; p.rows = rows; p.cols = cols; p.ld_src = ld;
  p.dst = nullptr; p.ld_dst = cols; p.dst_t = nullptr; p.ld_dst_t = rows;
  p.amax = nullptr; p.flag = nullptr; p.merge_amax = nullptr;
  p.colsum = scratch; p.telem_on_source = 1; p.tf32 = 0;
  p.vec_src = aligned16(dy, ld, esize(dy_dtype));
  p.vec_dst = 0; p.vec_dst_t = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = cast_dispatch(dy_dtype, work_dtype, p, s)) return st;
  launch_colsum_finalize(scratch, nparts, cols, work_dtype, db, accumulate, s);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}
