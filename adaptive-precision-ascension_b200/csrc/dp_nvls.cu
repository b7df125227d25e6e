// Data-parallel averaging of weight gradients through NVLink SHARP (NVLS),
// standalone form of the region protocol of dp_region.cuh, for gradients the
// weight-gradient GEMM did not reduce in its epilogue (split-K plans,
// accumulated gradients):
//
//   apa_dp_region_signal   after the gradient is written: publish every
//                          region of this rank (one multimem.red each)
//   apa_dp_region_reduce   a few CTAs: average the regions this rank owns
//                          (waits for every rank's signal, ld_reduce, st),
//                          or only those a split gradient left to it
//   apa_dp_region_wait     one thread: wait until every region of the
//                          gradient has been averaged, then advance the epoch
//
// Per GPU and gradient of B bytes the switch moves about B in and B out
// (the owned regions' sums and their multicast stores, and the reads other
// owners make of this rank's memory), independent of the number of ranks.
#include "dp_region.cuh"

namespace apa {
namespace dpnvls {

// defer_owned: also hand this rank's own regions to the side stream's
// pass over deferred regions (the caller runs no full reduce)
__global__ void region_signal_kernel(dpr::RegionArgs a, int defer_owned) {
  pdl_launch_dependents();
  pdl_wait();
  dpr::fence_sys();   // this rank's values (written by earlier kernels) before the signals
  const unsigned int tag = defer_owned ? *a.epoch + 1u : 0u;
  const int64_t n = dpr::num_regions(a.rows, a.cols);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (int64_t)gridDim.x * blockDim.x) {
    if (defer_owned && g % a.world == a.rank) a.deferred[g] = tag;
    dpr::signal_ready(a, g);
  }
}

__global__ void __launch_bounds__(256) region_reduce_kernel(dpr::RegionArgs a, int only_deferred) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned int epoch = *a.epoch;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t n = dpr::num_regions(a.rows, a.cols);
  const int ncb = dpr::region_cols(a.cols);
  // owned regions rank, rank + world, ... in order, one warp each
  for (int64_t g = a.rank + wid * a.world; g < n; g += warps * a.world) {
    if (only_deferred && *(volatile unsigned int*)(a.deferred + g) != epoch + 1u) continue;   // warp-uniform
    dpr::reduce_region(a, (int)(g / ncb), (int)(g % ncb), epoch, lane);
  }
}

__global__ void region_wait_kernel(const unsigned int* done, unsigned int* epoch, unsigned int regions) {
  const unsigned int e = *epoch + 1u;
  dpr::wait_at_least(done, regions * e, dpr::kStatusTimeoutDone);
  *epoch = e;
}

}  // namespace dpnvls

int dp_region_signal(const dpr::RegionArgs& a, int defer_owned, cudaStream_t s) {
  const int64_t n = dpr::num_regions(a.rows, a.cols);
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 64);
  return launch_kernel(dpnvls::region_signal_kernel, dim3(grid), dim3(256), 0, s, 1, a, defer_owned) == cudaSuccess
             ? APA_OK
             : APA_ERR_CUDA;
}

}  // namespace apa

extern "C" int apa_dp_regions(int64_t rows, int64_t cols, int64_t* regions_out) {
  if (!regions_out || rows <= 0 || cols <= 0 || rows >= (1ll << 31) || cols >= (1ll << 31)) return APA_ERR_INVALID;
  *regions_out = apa::dpr::num_regions((int)rows, (int)cols);
  return APA_OK;
}

extern "C" int apa_dp_region_signal(float* grad_mc, int64_t ld, int64_t rows, int64_t cols,
                                    const unsigned int* ready_local, unsigned int* ready_mc, unsigned int* done_mc,
                                    const unsigned int* epoch_local, unsigned int* deferred_local, int world, int rank,
                                    void* stream) {
  apa::dpr::RegionArgs a;
  if (int st = apa::dpr::make_region_args(&a, grad_mc, ld, rows, cols, ready_local, ready_mc, done_mc, epoch_local,
                                          deferred_local, world, rank))
    return st;
  return apa::dp_region_signal(a, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int apa_dp_region_reduce(float* grad_mc, int64_t ld, int64_t rows, int64_t cols,
                                    const unsigned int* ready_local, unsigned int* ready_mc, unsigned int* done_mc,
                                    const unsigned int* epoch_local, unsigned int* deferred_local, int world, int rank,
                                    int only_deferred, int ctas, void* stream) {
  apa::dpr::RegionArgs a;
  if (int st = apa::dpr::make_region_args(&a, grad_mc, ld, rows, cols, ready_local, ready_mc, done_mc, epoch_local,
                                          deferred_local, world, rank))
    return st;
  if (ctas < 1 || ctas > 1024 || (only_deferred != 0 && only_deferred != 1)) return APA_ERR_INVALID;
  return apa::launch_kernel(apa::dpnvls::region_reduce_kernel, dim3(ctas), dim3(256), 0,
                            static_cast<cudaStream_t>(stream), 1, a, only_deferred) == cudaSuccess
             ? APA_OK
             : APA_ERR_CUDA;
}

extern "C" int apa_dp_region_wait(const unsigned int* done_local, unsigned int* epoch_local, int64_t regions,
                                  void* stream) {
  if (!done_local || !epoch_local || regions <= 0 || regions >= (1ll << 31)) return APA_ERR_INVALID;
  // plain stream order: the wait depends on other GPUs only
  apa::dpnvls::region_wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(done_local, epoch_local,
                                                                                  (unsigned int)regions);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}
