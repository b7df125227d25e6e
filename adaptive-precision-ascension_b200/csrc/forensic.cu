// Device-side forensic statistics of one tensor (forensic mode,
// apa/layers.py:63-106 and manager.py:295-381 of the reference, which read
// every statistic back with .item()): max |x|, the flat index of the first
// element with that magnitude, the sum and the sum of squares, in one pass and
// with no host synchronisation. The record stays on the device until a
// forensic snapshot reads it.
//
// Record layout (five 8-byte words, zeroed by the launcher):
//   [0] key: (|x| as fp32 bits, NaN folded to one pattern) << 32 | ~index
//       (32-bit index), reduced with a 64-bit integer max: largest magnitude,
//       then smallest index
//   [1] sum (fp64)   [2] sum of squares (fp64)   [3] element count
//   [4] 1 if any element is NaN or infinite
#include "apa_common.cuh"

namespace apa {
namespace {

template <int DT>
__device__ __forceinline__ float stats_load(const void* p, int64_t i) {
  if constexpr (DT == APA_DT_F32) return static_cast<const float*>(p)[i];
  else if constexpr (DT == APA_DT_F16) return f16_to_f32(static_cast<const uint16_t*>(p)[i]);
  else if constexpr (DT == APA_DT_BF16) return bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
  else return e4m3_to_f32(static_cast<const uint8_t*>(p)[i]);
}

template <int DT>
__global__ void __launch_bounds__(256) tensor_stats_kernel(const void* src, int64_t n, unsigned long long* rec) {
  __shared__ unsigned long long s_key[8];
  __shared__ double s_sum[8], s_sq[8];
  __shared__ int s_bad[8];
  unsigned long long key = 0;
  double sum = 0.0, sq = 0.0;
  int bad = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = stats_load<DT>(src, i);
    uint32_t m = mag_bits(v);
    if (m > 0x7F800000u) m = 0x7FC00000u;   // every NaN ranks alike: the first one wins
    bad |= m >= 0x7F800000u ? 1 : 0;
    const unsigned long long k = ((unsigned long long)m << 32) | (unsigned long long)(~(uint32_t)i);
    key = k > key ? k : key;
    const double d = (double)v;
    sum += d;
    sq += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ok = __shfl_xor_sync(0xFFFFFFFFu, key, o);
    key = ok > key ? ok : key;
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
    sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
    bad |= __shfl_xor_sync(0xFFFFFFFFu, bad, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) { s_key[w] = key; s_sum[w] = sum; s_sq[w] = sq; s_bad[w] = bad; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int j = 1; j < 8; ++j) {
      key = s_key[j] > key ? s_key[j] : key;
      sum += s_sum[j];
      sq += s_sq[j];
      bad |= s_bad[j];
    }
    atomicMax(&rec[0], key);
    atomicAdd(reinterpret_cast<double*>(&rec[1]), sum);
    atomicAdd(reinterpret_cast<double*>(&rec[2]), sq);
    if (blockIdx.x == 0) rec[3] = (unsigned long long)n;
    if (bad) atomicMax(&rec[4], 1ull);
  }
}

}  // namespace
}  // namespace apa

extern "C" int apa_tensor_stats(const void* src, int dtype, int64_t n, unsigned long long* record, void* stream) {
  using namespace apa;
  if (!record || n < 0 || (n > 0 && !src)) return APA_ERR_INVALID;
  if (n >= (int64_t(1) << 32)) return APA_ERR_UNSUPPORTED;   // the index field is 32 bits
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(record, 0, 5 * sizeof(unsigned long long), s) != cudaSuccess) return APA_ERR_CUDA;
  if (n == 0) return APA_OK;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 4));
  switch (dtype) {
    case APA_DT_F32: tensor_stats_kernel<APA_DT_F32><<<grid, 256, 0, s>>>(src, n, record); break;
    case APA_DT_F16: tensor_stats_kernel<APA_DT_F16><<<grid, 256, 0, s>>>(src, n, record); break;
    case APA_DT_BF16: tensor_stats_kernel<APA_DT_BF16><<<grid, 256, 0, s>>>(src, n, record); break;
    case APA_DT_E4M3: tensor_stats_kernel<APA_DT_E4M3><<<grid, 256, 0, s>>>(src, n, record); break;
    default: return APA_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}
