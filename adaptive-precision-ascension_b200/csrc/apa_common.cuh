// Shared device helpers for the APA kernels (sm_100a only).
//
// Element conversions reproduce what torch does for the reference's casts
// (apa/layers.py:17-21 boundary cast, :370-372 working copy, and the autograd
// engine's re-casts of returned gradients). They are written from the format
// definitions (OCP FP8 E4M3, IEEE-754 binary16/bfloat16), not from any
// library's implementation.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "../../include/apa_kernels.h"

namespace apa {

// ---------------------------------------------------------------------------
// Status word shared by all kernels of the library: a bounded wait that gives
// up, or a launch that sees an impossible configuration, ORs a bit in here and
// returns instead of trapping. The host reads it with apa_get_device_status().
// ---------------------------------------------------------------------------
__device__ unsigned int g_status = 0;   // library is one translation unit

constexpr unsigned int kStatusTimeoutFull = 1u << 0;   // MMA waited too long for a TMA stage
constexpr unsigned int kStatusTimeoutEmpty = 1u << 1;  // producer waited too long for a free stage
constexpr unsigned int kStatusTimeoutAcc = 1u << 2;    // accumulator hand-off timed out
constexpr unsigned int kStatusBadConfig = 1u << 3;

constexpr unsigned long long kWaitLimitNs = 2000000000ull;   // 2 s

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch. The library launches its kernels with
// programmatic stream serialization, so the next kernel in a stream (or CUDA
// graph) can be scheduled while the current one finishes: every kernel lets
// its dependents launch as soon as all its CTAs are resident
// (pdl_launch_dependents) and, after a prologue that touches only shared and
// tensor memory and its parameters, waits in pdl_wait until the previous
// kernel has completed and its memory operations are visible, before it reads
// or writes global memory. Both instructions are no-ops for a launch without
// the attribute. A dependent can only start on resources the running kernels
// leave free, and only after every CTA of the kernel before it has started,
// so the early start cannot starve that kernel.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 1: launch with programmatic stream serialization (apa_set_pdl)
static int g_pdl = 1;

// cudaLaunchKernelEx with the library's launch attributes: programmatic
// stream serialization when enabled, and a cluster of `cluster_x` CTAs
// along x when cluster_x > 1.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                          int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned int n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (g_pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// E4M3 (float8_e4m3fn): bias 7, 3 mantissa bits, no infinities, S.1111.111 is
// NaN, largest finite 448. torch's conversion is non-saturating: the rounded
// magnitude 480 does not exist, so |x| > 464 (the midpoint between 448 and
// 480) and any Inf/NaN encode as NaN with the input's sign.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t e4m3_from_f32(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t s = (u >> 24) & 0x80u;
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x43E80000u) return s | 0x7Fu;          // > 464.0f, Inf or NaN
  if (a < 0x3C800000u) {                          // below 2^-6: one quantum 2^-9
    const float v = __uint_as_float(a) * 512.0f;  // exact power-of-two scaling
    return s | __float2uint_rn(v);                // round half to even; 8 encodes 2^-6
  }
  // normal range: keep sign-less exponent + 3 mantissa bits, round half to even
  uint32_t keep = a >> 20;
  const uint32_t rem = a & 0xFFFFFu;
  if (rem > 0x80000u || (rem == 0x80000u && (keep & 1u))) keep += 1u;
  return s | (keep - (120u << 3));                // re-bias exponent 127 -> 7
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t s = (b & 0x80u) << 24;
  const uint32_t e = (b >> 3) & 0xFu, m = b & 7u;
  if ((b & 0x7Fu) == 0x7Fu) return __uint_as_float(s | 0x7FC00000u);
  if (e == 0) return __uint_as_float(s | __float_as_uint((float)m * 0.001953125f));
  return __uint_as_float(s | ((e + 120u) << 23) | (m << 20));
}

// magnitude of an E4M3 code as fp32 bits (NaN sorts above every finite value)
__device__ __forceinline__ uint32_t e4m3_mag_bits(uint32_t b) {
  return __float_as_uint(e4m3_to_f32(b & 0x7Fu));
}

// ---------------------------------------------------------------------------
// binary16: IEEE round-to-nearest-even, overflow to +-Inf. A NaN keeps its sign
// and the top ten payload bits with the quiet bit set (torch's vectorised CPU
// conversion does the same; payload bits are not a parity target).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint16_t f16_from_f32(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u)
    return (uint16_t)(((u >> 16) & 0x8000u) | 0x7E00u | ((u >> 13) & 0x3FFu));
  return __half_as_ushort(__float2half_rn(f));
}

// binary16 -> fp32 is exact; a NaN keeps its sign and payload (the hardware
// conversion would return a canonical, sign-less NaN).
__device__ __forceinline__ float f16_to_f32(uint16_t h) {
  if ((h & 0x7C00u) == 0x7C00u && (h & 0x3FFu))
    return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7FC00000u | ((uint32_t)(h & 0x3FFu) << 13));
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t bf16_from_f32(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
  return __uint_as_float(((uint32_t)h) << 16);
}

// fp32 -> the TF32 operand grid (10 mantissa bits), round half to even,
// kept in fp32 storage. The tensor core reads only the top 19 bits of an fp32
// operand; rounding first halves the product error compared to dropping the
// low bits. Inf/NaN pass through.
__device__ __forceinline__ uint32_t tf32_rn_bits(uint32_t u) {
  if ((u & 0x7F800000u) == 0x7F800000u) return u;
  return (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
}

// E4M3 -> binary16 is exact; the NaN code keeps sign and mantissa (0x7F80).
__device__ __forceinline__ uint16_t e4m3_to_f16(uint32_t b) {
  if ((b & 0x7Fu) == 0x7Fu) return (uint16_t)(((b & 0x80u) << 8) | 0x7F80u);
  return f16_from_f32(e4m3_to_f32(b));
}

// ---------------------------------------------------------------------------
// Paired hardware conversions. The E4M3 one saturates (|x| > 448 -> 448, Inf
// -> 448, NaN -> NaN); callers apply the non-saturating rule of the reference
// (|x| > 464, Inf and NaN -> 0x7F | sign) wherever a value above 464 or a
// non-finite value can occur; below that the hardware's round-to-nearest-even
// equals e4m3_from_f32.
// ---------------------------------------------------------------------------
constexpr uint32_t kE4M3NaNThresholdBits = 0x43E80000u;   // 464.0f

// {lo, hi} -> 16 bits: lo's code in bits 0-7, hi's in bits 8-15 (saturating)
__device__ __forceinline__ uint32_t e4m3x2_sat(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// {lo, hi} -> 16 bits with the reference's non-saturating rule applied to both
__device__ __forceinline__ uint32_t e4m3x2_exact(float lo, float hi) {
  uint32_t r = e4m3x2_sat(lo, hi);
  const uint32_t ul = __float_as_uint(lo), uh = __float_as_uint(hi);
  if ((ul & 0x7FFFFFFFu) > kE4M3NaNThresholdBits) r = (r & 0xFF00u) | 0x7Fu | ((ul >> 24) & 0x80u);
  if ((uh & 0x7FFFFFFFu) > kE4M3NaNThresholdBits) r = (r & 0x00FFu) | 0x7F00u | ((uh >> 16) & 0x8000u);
  return r;
}

// two E4M3 codes (bits 0-7, 8-15) -> two binary16 values (exact) in one word
__device__ __forceinline__ uint32_t f16x2_from_e4m3x2(uint32_t codes) {
  uint32_t r;
  asm("{\n\t.reg .b16 t;\n\tmov.b16 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(r) : "h"((uint16_t)codes));
  return r;
}

// {lo, hi} fp32 -> binary16 pair (round to nearest even), lo in bits 0-15
__device__ __forceinline__ uint32_t f16x2_from_f32(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float f16lo_to_f32(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w & 0xFFFFu))); }
__device__ __forceinline__ float f16hi_to_f32(uint32_t w) { return __half2float(__ushort_as_half((uint16_t)(w >> 16))); }

// |v| as fp32 bits: comparing these as unsigned integers orders magnitudes
// with every NaN above +Inf, which is the NaN-propagating max torch.max uses.
__device__ __forceinline__ uint32_t mag_bits(float v) {
  return __float_as_uint(v) & 0x7FFFFFFFu;
}

__device__ __forceinline__ bool bits_nonfinite(uint32_t mag) { return mag >= 0x7F800000u; }

// Warp-level max of unsigned values.
__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Merge a block-reduced magnitude into a module's telemetry pair
// (gpu_amax: running NaN-propagating max; gpu_has_nonfinite: max with 1).
// amax holds non-negative floats or NaN, whose bit patterns order correctly
// as signed integers, so one integer atomicMax implements torch.maximum.
__device__ __forceinline__ void telem_commit(float* amax, int* flag, uint32_t mag) {
  if (amax) atomicMax(reinterpret_cast<int*>(amax), (int)mag);
  if (flag && bits_nonfinite(mag)) atomicMax(flag, 1);
}

}  // namespace apa
