// Data-parallel averaging of an fp32 weight gradient through NVLink SHARP,
// in regions: the gradient [rows, cols] (row pitch ld) lives in a symmetric
// allocation bound to a multicast object, and is cut into regions of 32 rows
// x 64 columns; region g = rb * ceil(cols / 64) + cb belongs to rank
// g % world. Every rank, once its own values of a region are in its memory,
// adds 1 to that region's ready counter on every rank (one multimem.red);
// the owner, once the counter shows all ranks, reads the region summed by the
// switch (multimem.ld_reduce), scales it by 1 / world and writes the mean to
// every rank (multimem.st), then adds 1 to every rank's done counter. A
// one-thread wait (apa_dp_region_wait) holds its stream until the done
// counter shows every region, then advances this rank's epoch.
//
// Counters only grow: in launch e (this rank's epoch word, read on the
// device) a region is ready at world x (e + 1) and the gradient is done at
// regions x (e + 1), so the launches replay from CUDA graphs unchanged.
//
// The weight-gradient GEMM runs the protocol in its epilogue (the reduction
// of finished regions overlaps the MMAs of later tiles); dp_nvls.cu has the
// same protocol as standalone kernels for gradients written some other way
// (a gradient split along the tokens marks its owned regions deferred, a
// local word per region tagged with the launch, for the standalone kernel a
// side stream runs after it). Every rank runs the same GEMMs in the same
// order, and every warp signals a tile's regions before it waits for any of
// them, so no wait depends on work queued behind another wait (every rank
// must produce every such gradient in every step; the host checks). Every
// wait is bounded (2 s); on expiry the waiter sets a status bit and still
// signals, so the other ranks' waits end, and later waits give up at once.
#pragma once

#include "apa_common.cuh"

namespace apa {
namespace dpr {

constexpr int kRegionRows = 32;
constexpr int kRegionCols = 64;
constexpr unsigned int kStatusTimeoutReady = 1u << 12;   // a region's contributions did not all arrive
constexpr unsigned int kStatusTimeoutDone = 1u << 13;    // the gradient's regions were not all reduced

// The gradient and its counters (all nullable when the reduction is off).
struct RegionArgs {
  float* mc;                       // multicast address of gradient element [0, 0]
  int64_t ld;                      // row pitch (elements; a multiple of 4)
  int rows, cols;
  unsigned int* ready_mc;          // per-region counters, multicast
  const unsigned int* ready;       // the same counters, this rank's copy
  unsigned int* done_mc;           // regions reduced, multicast
  const unsigned int* epoch;       // this rank's launch count for this gradient
  unsigned int* deferred;          // per region, this rank's copy: epoch + 1 when left to the side stream
  int world, rank;
  float scale;                     // 1 / world
};

__host__ __device__ __forceinline__ int region_cols(int cols) { return (cols + kRegionCols - 1) / kRegionCols; }
__host__ __device__ __forceinline__ int64_t num_regions(int rows, int cols) {
  return (int64_t)((rows + kRegionRows - 1) / kRegionRows) * region_cols(cols);
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_add_release(unsigned int* mc, unsigned int v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ float4 ld_reduce4(const float* mc) {
  float4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}

__device__ __forceinline__ void st4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

// A data-parallel wait of this library expired and the status word has not
// been cleared since: the ranks are out of step, and every later wait gives
// up at once instead of adding its own 2 s (a gradient has thousands of
// regions).
__device__ __forceinline__ bool dp_failed() {
  return (*(volatile unsigned int*)&g_status & (kStatusTimeoutReady | kStatusTimeoutDone)) != 0u;
}

// One thread: wait until *p >= target (wrapping compare), at most 2 s.
__device__ __forceinline__ bool wait_at_least(const unsigned int* p, unsigned int target, unsigned int why) {
  if ((int)(ld_acquire_sys(p) - target) >= 0) return true;
  if (dp_failed()) return false;
  const unsigned long long t0 = global_ns();
  while ((int)(ld_acquire_sys(p) - target) < 0) {
    if (global_ns() - t0 > kWaitLimitNs || dp_failed()) {
      atomicOr(&g_status, why);
      return false;
    }
  }
  return true;
}


// One thread, after this rank's values of region g are globally visible.
__device__ __forceinline__ void signal_ready(const RegionArgs& a, int64_t g) { red_add_release(a.ready_mc + g, 1u); }

// One warp, owner of region (rb, cb) in launch `epoch`: wait for every
// rank's values, average the region across ranks, tell every rank.
__device__ __forceinline__ void reduce_region(const RegionArgs& a, int rb, int cb, unsigned int epoch, int lane) {
  const int64_t g = (int64_t)rb * region_cols(a.cols) + cb;
  int ok = 1;
  if (lane == 0) ok = wait_at_least(a.ready + g, (unsigned int)a.world * (epoch + 1u), kStatusTimeoutReady) ? 1 : 0;
  ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
  fence_sys();
  if (ok) {
    // half a warp per row: 16 lanes x 4 columns = the region's 64 columns;
    // two halves of 16 rows, each with all eight of a lane's loads issued
    // before its first store
    constexpr int kPer = kRegionRows / 4;
    const int r_in = lane >> 4, c = cb * kRegionCols + (lane & 15) * 4;
    const bool col_ok = c < a.cols;   // cols is a multiple of 4
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      const int r0 = rb * kRegionRows + h * (kRegionRows / 2);
      float4 v[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int r = r0 + 2 * i + r_in;
        if (col_ok && r < a.rows) v[i] = ld_reduce4(a.mc + (int64_t)r * a.ld + c);
      }
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int r = r0 + 2 * i + r_in;
        if (col_ok && r < a.rows) {
          v[i].x *= a.scale;
          v[i].y *= a.scale;
          v[i].z *= a.scale;
          v[i].w *= a.scale;
          st4(a.mc + (int64_t)r * a.ld + c, v[i]);
        }
      }
    }
  }
  fence_sys();
  __syncwarp();
  if (lane == 0) red_add_release(a.done_mc, 1u);   // also after a timeout, so the waits of every rank end
}

// Validated RegionArgs for the C-ABI entry points.
inline int make_region_args(RegionArgs* a, float* grad_mc, int64_t ld, int64_t rows, int64_t cols,
                            const unsigned int* ready_local, unsigned int* ready_mc, unsigned int* done_mc,
                            const unsigned int* epoch_local, unsigned int* deferred_local, int world, int rank) {
  if (!grad_mc || !ready_local || !ready_mc || !done_mc || !epoch_local || !deferred_local) return APA_ERR_INVALID;
  if (rows <= 0 || cols <= 0 || rows >= (1ll << 31) || cols >= (1ll << 31) || ld < cols) return APA_ERR_INVALID;
  if (world < 2 || world > 64 || rank < 0 || rank >= world) return APA_ERR_INVALID;
  if ((cols & 3) != 0 || (ld & 3) != 0) return APA_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(grad_mc) & 15u) != 0) return APA_ERR_ALIGN;
  a->mc = grad_mc; a->ld = ld; a->rows = (int)rows; a->cols = (int)cols;
  a->ready_mc = ready_mc; a->ready = ready_local; a->done_mc = done_mc; a->epoch = epoch_local;
  a->deferred = deferred_local;
  a->world = world; a->rank = rank; a->scale = 1.0f / (float)world;
  return APA_OK;
}

}  // namespace dpr
}  // namespace apa
