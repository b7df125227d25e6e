// Data-parallel averaging of weight gradients through NVLink SHARP (NVLS):
// every rank's fp32 gradient lives in one buffer of a symmetric allocation
// bound to an NVLink multicast object; each rank averages its 1/world shard
// of every gradient with multimem.ld_reduce (the switch sums the ranks'
// copies) and writes the mean back to all ranks with one multimem.st.
//
// Per gradient and step, three launches on the caller's streams:
//   apa_dp_signal     1 thread, after the weight-gradient GEMM: release this
//                     rank's gradient and add 1 to every rank's `ready` word
//                     (one multimem.red through the switch).
//   apa_dp_allreduce  a few CTAs: wait until `ready` reaches world x epoch
//                     (every rank's gradient is complete), average this
//                     rank's shard, then add 1 to every rank's `done` word.
//   apa_dp_wait       1 thread: wait until `done` reaches world x ctas x
//                     epoch (every shard of this gradient has been written on
//                     this rank), then advance this rank's epoch.
// Epochs are device words read and advanced by the kernels themselves, so the
// launches can be replayed from a CUDA graph. No kernel waits on another
// kernel of its own GPU: the signal and the local reduce precede the waits
// that depend on them in stream order, and the waits depend only on the
// other GPUs' kernels. Every wait is bounded (2 s of %globaltimer); on expiry
// the kernel sets a bit in the library status word and returns.
//
// Per GPU and gradient of B bytes the switch moves B / world in (the reduced
// shard) and B / world out (the multicast store), against 2 (world-1)/world B
// in and out for a ring all-reduce.
#include "apa_common.cuh"

namespace apa {
namespace dpnvls {

constexpr unsigned int kStatusTimeoutReady = 1u << 12;
constexpr unsigned int kStatusTimeoutDone = 1u << 13;

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void mc_red_add_release(unsigned int* mc, unsigned int v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

__device__ __forceinline__ float4 mc_ld_reduce_f32x4(const float* mc) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

__device__ __forceinline__ void mc_st_f32x4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

// Wait (one thread) until *p >= target, at most kWaitLimitNs; false on expiry.
__device__ __forceinline__ bool wait_at_least(const unsigned int* p, unsigned int target, unsigned int why) {
  if ((int)(ld_acquire_sys(p) - target) >= 0) return true;
  const unsigned long long t0 = global_ns();
  while ((int)(ld_acquire_sys(p) - target) < 0) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_status, why);
      return false;
    }
  }
  return true;
}

__global__ void signal_kernel(unsigned int* mc_ready) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  mc_red_add_release(mc_ready, 1u);
}

// ready_local / epoch_local: this rank's words; mc_grad / mc_done: multicast
// addresses. n4: float4 elements of the gradient; the shard of rank r is
// float4s [r * per, min((r + 1) * per, n4)).
__global__ void __launch_bounds__(512) allreduce_kernel(float* mc_grad, int64_t n4, int world, int rank,
                                                        const unsigned int* ready_local, unsigned int* mc_done,
                                                        const unsigned int* epoch_local, float inv_world) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const unsigned int target = (unsigned int)world * (*epoch_local + 1u);
    s_ok = wait_at_least(ready_local, target, kStatusTimeoutReady) ? 1 : 0;
  }
  __syncthreads();
  if (s_ok) {
    // kIlp independent reductions in flight per thread: one multimem load
    // crosses the switch and back, so a thread with a single outstanding load
    // leaves the CTAs latency-bound far below the link rate
    constexpr int kIlp = 8;
    const int64_t per = (n4 + world - 1) / world;
    const int64_t lo = (int64_t)rank * per;
    const int64_t hi = lo + per < n4 ? lo + per : n4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < hi; base += kIlp * stride) {
      float4 v[kIlp];
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        const int64_t i = base + u * stride;
        if (i < hi) v[u] = mc_ld_reduce_f32x4(mc_grad + 4 * i);
      }
#pragma unroll
      for (int u = 0; u < kIlp; ++u) {
        const int64_t i = base + u * stride;
        if (i < hi) {
          v[u].x *= inv_world;
          v[u].y *= inv_world;
          v[u].z *= inv_world;
          v[u].w *= inv_world;
          mc_st_f32x4(mc_grad + 4 * i, v[u]);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // every CTA signals, also after a timeout, so the other ranks' waits end
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    mc_red_add_release(mc_done, 1u);
  }
}

__global__ void wait_kernel(const unsigned int* done_local, unsigned int* epoch_local, int world, int ctas) {
  const unsigned int e = *epoch_local + 1u;
  wait_at_least(done_local, (unsigned int)world * (unsigned int)ctas * e, kStatusTimeoutDone);
  *epoch_local = e;
}

}  // namespace dpnvls
}  // namespace apa

namespace {
bool dp_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

extern "C" int apa_dp_signal(unsigned int* mc_ready, void* stream) {
  if (!mc_ready) return APA_ERR_INVALID;
  apa::dpnvls::signal_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(mc_ready);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_dp_allreduce(float* mc_grad, int64_t n, int world, int rank, const unsigned int* ready_local,
                                unsigned int* mc_done, const unsigned int* epoch_local, int ctas, void* stream) {
  if (!mc_grad || !ready_local || !mc_done || !epoch_local || n <= 0 || (n & 3) != 0 || world < 2 || world > 64 ||
      rank < 0 || rank >= world || ctas < 1 || ctas > 1024)
    return APA_ERR_INVALID;
  if (!dp_aligned16(mc_grad)) return APA_ERR_ALIGN;
  apa::dpnvls::allreduce_kernel<<<ctas, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      mc_grad, n / 4, world, rank, ready_local, mc_done, epoch_local, 1.0f / (float)world);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_dp_wait(const unsigned int* done_local, unsigned int* epoch_local, int world, int ctas,
                           void* stream) {
  if (!done_local || !epoch_local || world < 2 || ctas < 1) return APA_ERR_INVALID;
  apa::dpnvls::wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(done_local, epoch_local, world, ctas);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}
