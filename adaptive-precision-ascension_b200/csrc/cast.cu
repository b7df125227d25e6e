// K1: cast + telemetry kernels (HBM-bound).
//
// One pass over a [rows, cols] matrix converts every element to the working
// dtype (the reference's boundary cast, apa/layers.py:17-21, and working-copy
// refresh, :370-372), optionally writes the transposed copy the backward GEMMs
// consume as a K-major operand, optionally writes per-64-row column partial
// sums (bias gradient, layers.py:239-241/265-266/274-275), and folds
// max|value| / NaN-Inf detection into the module's telemetry buffers
// (apa/telemetry.py:7-21) so no separate reduction pass reads HBM.
#include "apa_common.cuh"

namespace apa {

static int g_num_sms = 0;

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

int esize(int dt) {
  switch (dt) {
    case APA_DT_F32: return 4;
    case APA_DT_F16: case APA_DT_BF16: return 2;
    case APA_DT_E4M3: return 1;
    default: return 0;
  }
}

bool aligned16(const void* p, int64_t ld, int es) {
  return p == nullptr || ((reinterpret_cast<uintptr_t>(p) & 15u) == 0 && ((ld * es) & 15) == 0);
}


namespace {

constexpr int kTile = 64;          // 64 x 64 element tile per iteration
constexpr int kThreads = 256;      // 4 threads per tile row, 16 elements each
constexpr int kSeg = 16;

template <int DT> struct Elem;
template <> struct Elem<APA_DT_F32> { using T = float; static constexpr int bytes = 4; };
template <> struct Elem<APA_DT_F16> { using T = uint16_t; static constexpr int bytes = 2; };
template <> struct Elem<APA_DT_BF16> { using T = uint16_t; static constexpr int bytes = 2; };
template <> struct Elem<APA_DT_E4M3> { using T = uint8_t; static constexpr int bytes = 1; };

template <int DT>
__device__ __forceinline__ float load_as_f32(const void* p, int64_t i) {
  if constexpr (DT == APA_DT_F32) return static_cast<const float*>(p)[i];
  else if constexpr (DT == APA_DT_F16) return f16_to_f32(static_cast<const uint16_t*>(p)[i]);
  else if constexpr (DT == APA_DT_BF16) return bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
  else return e4m3_to_f32(static_cast<const uint8_t*>(p)[i]);
}

// Encode an fp32 value (exactly representable in SRC) as DST bits.
template <int SRC, int DST>
__device__ __forceinline__ uint32_t encode(float v) {
  if constexpr (DST == APA_DT_E4M3) return e4m3_from_f32(v);
  else if constexpr (DST == APA_DT_F16) {
    if constexpr (SRC == APA_DT_F16) return f16_from_f32(v);  // identity on values
    else return f16_from_f32(v);
  } else if constexpr (DST == APA_DT_BF16) return bf16_from_f32(v);
  else return __float_as_uint(v);
}

template <int DST>
__device__ __forceinline__ float decode(uint32_t c) {
  if constexpr (DST == APA_DT_E4M3) return e4m3_to_f32(c);
  else if constexpr (DST == APA_DT_F16) return f16_to_f32((uint16_t)c);
  else if constexpr (DST == APA_DT_BF16) return bf16_to_f32((uint16_t)c);
  else return __uint_as_float(c);
}

template <int DST>
__device__ __forceinline__ uint32_t code_mag_bits(uint32_t c) {
  if constexpr (DST == APA_DT_E4M3) return e4m3_mag_bits(c);
  else return mag_bits(decode<DST>(c));
}

template <int DST>
__device__ __forceinline__ void store_code(void* base, int64_t i, uint32_t c) {
  if constexpr (Elem<DST>::bytes == 1) static_cast<uint8_t*>(base)[i] = (uint8_t)c;
  else if constexpr (Elem<DST>::bytes == 2) static_cast<uint16_t*>(base)[i] = (uint16_t)c;
  else static_cast<uint32_t*>(base)[i] = c;
}

// Store 16 consecutive codes starting at element i (16-byte aligned when vec).
template <int DST>
__device__ __forceinline__ void store16(void* base, int64_t i, const uint32_t (&c)[kSeg], bool vec) {
  if (vec) {
    if constexpr (Elem<DST>::bytes == 1) {
      uint4 w;
      w.x = c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24);
      w.y = c[4] | (c[5] << 8) | (c[6] << 16) | (c[7] << 24);
      w.z = c[8] | (c[9] << 8) | (c[10] << 16) | (c[11] << 24);
      w.w = c[12] | (c[13] << 8) | (c[14] << 16) | (c[15] << 24);
      *reinterpret_cast<uint4*>(static_cast<uint8_t*>(base) + i) = w;
    } else if constexpr (Elem<DST>::bytes == 2) {
      uint4* p = reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + i);
#pragma unroll
      for (int q = 0; q < 2; ++q)
        p[q] = make_uint4(c[8 * q + 0] | (c[8 * q + 1] << 16), c[8 * q + 2] | (c[8 * q + 3] << 16),
                          c[8 * q + 4] | (c[8 * q + 5] << 16), c[8 * q + 6] | (c[8 * q + 7] << 16));
    } else {
      uint4* p = reinterpret_cast<uint4*>(static_cast<uint32_t*>(base) + i);
#pragma unroll
      for (int q = 0; q < 4; ++q) p[q] = make_uint4(c[4 * q], c[4 * q + 1], c[4 * q + 2], c[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kSeg; ++j) store_code<DST>(base, i + j, c[j]);
  }
}

struct CastParams {
  const void* src; int64_t rows, cols, ld_src;
  void* dst; int64_t ld_dst;
  void* dst_t; int64_t ld_dst_t;
  float* amax; int* flag;
  const float* merge_amax;
  float* colsum;          // [ceil(rows/64), cols] partial sums of the cast values
  int telem_on_source;
  int vec_src, vec_dst, vec_dst_t;
  int tf32;               // DST fp32 only: stored operands rounded to TF32
};

template <int SRC, int DST>
__global__ void __launch_bounds__(kThreads, 4) cast_kernel(CastParams p) {
  pdl_launch_dependents();
  pdl_wait();
  // 64 x 64 tile per iteration; thread t owns the 4 x 4 block at rows 4a..4a+3,
  // columns 4b..4b+3 (a = t / 16, b = t % 16). The transposed copy goes
  // through shared memory as packed column strips of 4 codes.
  constexpr int ES = Elem<DST>::bytes;
  constexpr int PITCH = 64 * ES + 4;   // bytes per transposed row; the 4-byte pad spreads banks
  __shared__ __align__(16) uint8_t tileT[64 * PITCH];
  __shared__ float csum_s[8][64];
  __shared__ uint32_t red[kThreads / 32];
  const int t = threadIdx.x;
  const int a = t >> 4, b = t & 15;
  const int warp = t >> 5, lane = t & 31;
  const int64_t tiles_r = (p.rows + kTile - 1) / kTile;
  const int64_t tiles_c = (p.cols + kTile - 1) / kTile;
  const int64_t ntiles = tiles_r * tiles_c;
  const bool stage = (p.dst_t != nullptr) || (p.colsum != nullptr);
  uint32_t msrc = 0;   // max |source value| (fp32 bits) over in-bounds elements

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t tr = tile / tiles_c, tc = tile - tr * tiles_c;
    const int64_t r0 = tr * kTile + 4 * a;
    const int64_t c0 = tc * kTile + 4 * b;
    const bool cols_full = c0 + 4 <= p.cols;
    float v[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = r0 + i;
      const bool row_ok = row < p.rows;
      if (row_ok && cols_full && p.vec_src) {
        const int64_t off = row * p.ld_src + c0;
        if constexpr (Elem<SRC>::bytes == 4) {
          const float4 w = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.src) + off));
          v[i][0] = w.x; v[i][1] = w.y; v[i][2] = w.z; v[i][3] = w.w;
        } else {
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.src) + off));
          const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if constexpr (SRC == APA_DT_BF16) {
              v[i][2 * h] = bf16_to_f32((uint16_t)(ws[h] & 0xFFFFu));
              v[i][2 * h + 1] = bf16_to_f32((uint16_t)(ws[h] >> 16));
            } else {
              v[i][2 * h] = f16_to_f32((uint16_t)(ws[h] & 0xFFFFu));
              v[i][2 * h + 1] = f16_to_f32((uint16_t)(ws[h] >> 16));
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[i][j] = (row_ok && c0 + j < p.cols) ? load_as_f32<SRC>(p.src, row * p.ld_src + c0 + j) : 0.0f;
      }
    }
    // telemetry on the source magnitudes (out-of-bounds slots hold +0)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) msrc = max(msrc, mag_bits(v[i][j]));

    // encode
    uint32_t code[4][4];
    if constexpr (DST == APA_DT_E4M3) {
      uint32_t m = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) m = max(m, mag_bits(v[i][j]));
      const bool big = m > kE4M3NaNThresholdBits;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          const uint32_t w = big ? e4m3x2_exact(v[i][j], v[i][j + 1]) : e4m3x2_sat(v[i][j], v[i][j + 1]);
          code[i][j] = w & 0xFFu;
          code[i][j + 1] = w >> 8;
        }
    } else if constexpr (DST == APA_DT_F16) {
      uint32_t m = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) m = max(m, mag_bits(v[i][j]));
      if (m > 0x7F800000u) {   // a NaN: keep its sign and payload as torch does
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) code[i][j] = f16_from_f32(v[i][j]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; j += 2) {
            const uint32_t w = f16x2_from_f32(v[i][j], v[i][j + 1]);
            code[i][j] = w & 0xFFFFu;
            code[i][j + 1] = w >> 16;
          }
      }
    } else if constexpr (DST == APA_DT_BF16) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) code[i][j] = bf16_from_f32(v[i][j]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) code[i][j] = __float_as_uint(v[i][j]);
    }

    // row-major copy (TF32 operands rounded on the way out)
    if (p.dst) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t row = r0 + i;
        if (row >= p.rows) continue;
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (DST == APA_DT_F32) o[j] = p.tf32 ? tf32_rn_bits(code[i][j]) : code[i][j];
          else o[j] = code[i][j];
        }
        const int64_t off = row * p.ld_dst + c0;
        if (cols_full && p.vec_dst) {
          if constexpr (ES == 1)
            *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(p.dst) + off) = o[0] | (o[1] << 8) | (o[2] << 16) | (o[3] << 24);
          else if constexpr (ES == 2)
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.dst) + off) = make_uint2(o[0] | (o[1] << 16), o[2] | (o[3] << 16));
          else
            *reinterpret_cast<uint4*>(static_cast<uint32_t*>(p.dst) + off) = make_uint4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (c0 + j < p.cols) store_code<DST>(p.dst, off + j, o[j]);
        }
      }
    }

    if (stage) {
      // column strips: codes of rows 4a..4a+3 of column 4b+c, packed, at
      // transposed row (4b + c), byte offset 4a*ES
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint8_t* dstT = tileT + (4 * b + c) * PITCH + 4 * a * ES;
        if constexpr (ES == 1) {
          *reinterpret_cast<uint32_t*>(dstT) =
              code[0][c] | (code[1][c] << 8) | (code[2][c] << 16) | (code[3][c] << 24);
        } else if constexpr (ES == 2) {
          reinterpret_cast<uint32_t*>(dstT)[0] = code[0][c] | (code[1][c] << 16);
          reinterpret_cast<uint32_t*>(dstT)[1] = code[2][c] | (code[3][c] << 16);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) reinterpret_cast<uint32_t*>(dstT)[i] = code[i][c];
        }
      }
      if (p.colsum) {
        // partial column sums of the cast values over this thread's 4 rows,
        // then over the 16 threads sharing b (lanes b and b+16 of each warp,
        // then the 8 warps in a fixed order)
        float cs[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float s = 0.0f;
#pragma unroll
          for (int i = 0; i < 4; ++i) s += decode<DST>(code[i][c]);
          cs[c] = s + __shfl_xor_sync(0xFFFFFFFFu, s, 16);
        }
        if (lane < 16) {
#pragma unroll
          for (int c = 0; c < 4; ++c) csum_s[warp][4 * b + c] = cs[c];
        }
      }
      __syncthreads();
      if (p.colsum && t < 64) {
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) s += csum_s[w][t];
        const int64_t col = tc * kTile + t;
        if (col < p.cols) p.colsum[tr * p.cols + col] = s;
      }
      if (p.dst_t) {
        // transposed rows: 64 x (64*ES bytes) = 256*ES chunks of 16 bytes
#pragma unroll
        for (int k = 0; k < ES; ++k) {
          const int id = t + kThreads * k;
          const int j = id / (4 * ES);           // transposed row in the tile (source column)
          const int ch = id - j * (4 * ES);      // 16-byte chunk within that row
          const int64_t orow = tc * kTile + j;
          if (orow >= p.cols) continue;
          const uint32_t* s = reinterpret_cast<const uint32_t*>(tileT + j * PITCH + ch * 16);
          uint32_t w[4] = {s[0], s[1], s[2], s[3]};
          if constexpr (DST == APA_DT_F32) {
            if (p.tf32) {
#pragma unroll
              for (int h = 0; h < 4; ++h) w[h] = tf32_rn_bits(w[h]);
            }
          }
          constexpr int PER = 16 / ES;            // elements per chunk
          const int64_t ocol = tr * kTile + ch * PER;
          const int64_t off = orow * p.ld_dst_t + ocol;
          if (ocol + PER <= p.rows && p.vec_dst_t) {
            *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.dst_t) + off * ES) = make_uint4(w[0], w[1], w[2], w[3]);
          } else {
#pragma unroll
            for (int e = 0; e < PER; ++e) {
              if (ocol + e < p.rows) {
                uint32_t cval;
                if constexpr (ES == 1) cval = (w[e >> 2] >> (8 * (e & 3))) & 0xFFu;
                else if constexpr (ES == 2) cval = (w[e >> 1] >> (16 * (e & 1))) & 0xFFFFu;
                else cval = w[e];
                store_code<DST>(p.dst_t, off + e, cval);
              }
            }
          }
        }
      }
      __syncthreads();
    }
  }
  // telemetry: the cast values' max is the cast of the source max (rounding
  // to E4M3 / fp16 is monotone in magnitude, NaN rule included)
  uint32_t mag = msrc;
  if (!p.telem_on_source) {
    if constexpr (DST == APA_DT_E4M3) mag = e4m3_mag_bits(e4m3_from_f32(__uint_as_float(msrc)));
    else if constexpr (DST == APA_DT_F16) mag = mag_bits(f16_to_f32(f16_from_f32(__uint_as_float(msrc))));
    else if constexpr (DST == APA_DT_BF16) mag = mag_bits(bf16_to_f32(bf16_from_f32(__uint_as_float(msrc))));
  }
  mag = warp_max_u32(mag);
  if (lane == 0) red[warp] = mag;
  __syncthreads();
  if (t < 32) {
    uint32_t m = t < kThreads / 32 ? red[t] : 0u;
    m = warp_max_u32(m);
    if (t == 0) {
      telem_commit(p.amax, p.flag, m);
      if (blockIdx.x == 0 && p.merge_amax) telem_commit(p.amax, p.flag, mag_bits(*p.merge_amax));
    }
  }
}

// amax / nonfinite over a flat array (torch's track_telemetry_on_tensor on
// tensors no fused kernel produced: non-APA module gradients, manual calls).
template <int DT>
__global__ void __launch_bounds__(256) amax_kernel(const void* src, int64_t n, float* amax, int* flag, int vec) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ uint32_t red[8];
  uint32_t mag = 0;
  constexpr int per = 16 / Elem<DT>::bytes;
  const int64_t nvec = vec ? n / per : 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(src) + i);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      if constexpr (DT == APA_DT_F32) mag = max(mag, ws[h] & 0x7FFFFFFFu);
      else if constexpr (DT == APA_DT_F16) {
        mag = max(mag, mag_bits(f16_to_f32((uint16_t)(ws[h] & 0xFFFF))));
        mag = max(mag, mag_bits(f16_to_f32((uint16_t)(ws[h] >> 16))));
      } else if constexpr (DT == APA_DT_BF16) {
        mag = max(mag, mag_bits(bf16_to_f32((uint16_t)(ws[h] & 0xFFFF))));
        mag = max(mag, mag_bits(bf16_to_f32((uint16_t)(ws[h] >> 16))));
      } else {
#pragma unroll
        for (int b = 0; b < 4; ++b) mag = max(mag, e4m3_mag_bits((ws[h] >> (8 * b)) & 0xFF));
      }
    }
  }
  for (int64_t i = nvec * per + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    mag = max(mag, mag_bits(load_as_f32<DT>(src, i)));
  mag = warp_max_u32(mag);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mag;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t m = threadIdx.x < 8 ? red[threadIdx.x] : 0u;
    m = warp_max_u32(m);
    if (threadIdx.x == 0) telem_commit(amax, flag, m);
  }
}

// compute_underflow_ratio (telemetry.py:23-39) over a flat array: per-block
// counts of nonzero and below-threshold magnitudes, then the last block to
// finish turns them into the fp32 ratio (0 when nothing is nonzero) and
// either stores it or folds it into a running max (layers.py:404-407).
template <int DT>
__global__ void __launch_bounds__(256) underflow_kernel(const void* src, int64_t n, float vmin,
                                                        unsigned long long* counters, float* ratio_out,
                                                        int running_max) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ unsigned int s_nz[8], s_uf[8];
  const uint32_t vbits = __float_as_uint(vmin);
  unsigned int nz = 0, uf = 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint32_t m = mag_bits(load_as_f32<DT>(src, i));
    const bool nonzero = m != 0u && m <= 0x7F800000u;
    nz += nonzero;
    uf += (nonzero && m < vbits);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nz += __shfl_xor_sync(0xFFFFFFFFu, nz, o);
    uf += __shfl_xor_sync(0xFFFFFFFFu, uf, o);
  }
  if ((threadIdx.x & 31) == 0) { s_nz[threadIdx.x >> 5] = nz; s_uf[threadIdx.x >> 5] = uf; }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long bnz = 0, buf = 0;
    for (int w = 0; w < 8; ++w) { bnz += s_nz[w]; buf += s_uf[w]; }
    if (bnz) atomicAdd(&counters[0], bnz);
    if (buf) atomicAdd(&counters[1], buf);
    __threadfence();
    const unsigned long long ticket = atomicAdd(&counters[2], 1ull);
    if (ticket == (unsigned long long)gridDim.x - 1ull) {
      __threadfence();
      const unsigned long long tnz = atomicAdd(&counters[0], 0ull);
      const unsigned long long tuf = atomicAdd(&counters[1], 0ull);
      const float ratio = tnz ? __fdiv_rn(__ull2float_rn(tuf), __ull2float_rn(tnz)) : 0.0f;
      if (running_max) {
        const float old = *ratio_out;
        *ratio_out = (old != old) ? old : fmaxf(old, ratio);
      } else {
        *ratio_out = ratio;
      }
      counters[0] = 0ull; counters[1] = 0ull; counters[2] = 0ull;
    }
  }
}

// Bias gradient: sum the per-64-row partials in a fixed order, round to the
// working dtype (the autograd engine's cast to bias_work's dtype) and widen
// to fp32 for bias_master.grad (manager.py:200-204).
constexpr int kColsumWarps = 32;
__global__ void __launch_bounds__(kColsumWarps * 32) colsum_finalize_kernel(const float* partial, int64_t nparts,
                                                                           int64_t cols, int work_dt, float* out,
                                                                           int accumulate) {
  pdl_launch_dependents();
  pdl_wait();
  // block: 32 columns x 32 warps; warp w sums partial rows w, w+32, ... in
  // order (eight loads in flight), then warp 0 adds the 32 warp sums in order
  // (deterministic)
  __shared__ float part[kColsumWarps][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float s = 0.0f;
  if (c < cols) {
    int64_t r = w;
    for (; r + 7 * kColsumWarps < nparts; r += 8 * kColsumWarps) {
      float v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = partial[(r + k * kColsumWarps) * cols + c];
#pragma unroll
      for (int k = 0; k < 8; ++k) s += v[k];
    }
    for (; r < nparts; r += kColsumWarps) s += partial[r * cols + c];
  }
  part[w][lane] = s;
  __syncthreads();
  if (w == 0 && c < cols) {
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < kColsumWarps; ++k) t += part[k][lane];
    float q;
    if (work_dt == APA_DT_E4M3) q = e4m3_to_f32(e4m3_from_f32(t));
    else if (work_dt == APA_DT_F16) q = f16_to_f32(f16_from_f32(t));
    else q = t;
    out[c] = accumulate ? out[c] + q : q;
  }
}

void launch_colsum_finalize(const float* partial, int64_t nparts, int64_t cols, int work_dt, float* out,
                            int accumulate, cudaStream_t s) {
  const unsigned grid = (unsigned)((cols + 31) / 32);
  launch_kernel(colsum_finalize_kernel, dim3(grid), dim3(kColsumWarps * 32), 0, s, 1, partial, nparts, cols, work_dt,
                out, accumulate);
}

// Zero a list of int32 words (per-step flag reset, manager.py:161-168).
__global__ void zero_list_kernel(int* const* ptrs, int n) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) *ptrs[i] = 0;
}

template <int SRC, int DST>
int launch_cast_t(CastParams& p, cudaStream_t s) {
  const int64_t tiles = ((p.rows + kTile - 1) / kTile) * ((p.cols + kTile - 1) / kTile);
  int64_t grid = std::min<int64_t>(tiles, (int64_t)num_sms() * 4);
  if (grid < 1) grid = 1;
  if (launch_kernel(cast_kernel<SRC, DST>, dim3((unsigned)grid), dim3(kThreads), 0, s, 1, p) != cudaSuccess)
    return APA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

template <int SRC>
int launch_cast_dst(int dst_dt, CastParams& p, cudaStream_t s) {
  switch (dst_dt) {
    case APA_DT_E4M3: return launch_cast_t<SRC, APA_DT_E4M3>(p, s);
    case APA_DT_F16: return launch_cast_t<SRC, APA_DT_F16>(p, s);
    case APA_DT_F32: return launch_cast_t<SRC, APA_DT_F32>(p, s);
    case APA_DT_BF16: return launch_cast_t<SRC, APA_DT_BF16>(p, s);
    default: return APA_ERR_UNSUPPORTED;
  }
}

}  // namespace

// streaming TMA version for the aligned E4M3 / fp16 layouts (cast_tma.cu)
int cast_tma_try(int src_dt, int dst_dt, const CastParams& p, cudaStream_t s);

int cast_dispatch(int src_dt, int dst_dt, CastParams& p, cudaStream_t s) {
  switch (src_dt) {
    case APA_DT_F32: return launch_cast_dst<APA_DT_F32>(dst_dt, p, s);
    case APA_DT_BF16: return launch_cast_dst<APA_DT_BF16>(dst_dt, p, s);
    case APA_DT_F16: return launch_cast_dst<APA_DT_F16>(dst_dt, p, s);
    default: return APA_ERR_UNSUPPORTED;
  }
}

}  // namespace apa

using namespace apa;

extern "C" int apa_cast(const void* src, int src_dtype, int64_t rows, int64_t cols, int64_t ld_src,
                        void* dst, int dst_dtype, int64_t ld_dst, void* dst_t, int64_t ld_dst_t,
                        float* amax, int32_t* flag, int telem_on_source, const float* merge_amax,
                        float* colsum_partial, void* stream) {
  if (!src || rows < 0 || cols < 0 || ld_src < cols) return APA_ERR_INVALID;
  if (dst && ld_dst < cols) return APA_ERR_INVALID;
  if (dst_t && ld_dst_t < rows) return APA_ERR_INVALID;
  const int tf32 = dst_dtype == APA_DT_TF32;
  if (tf32) dst_dtype = APA_DT_F32;
  const int es_src = esize(src_dtype), es_dst = esize(dst_dtype);
  if (!es_src || !es_dst || src_dtype == APA_DT_E4M3) return APA_ERR_UNSUPPORTED;
  if (rows == 0 || cols == 0) {
    if (merge_amax) return apa_merge_telemetry(amax, flag, merge_amax, stream);
    return APA_OK;
  }
  CastParams p;
  p.src = src; p.rows = rows; p.cols = cols; p.ld_src = ld_src;
  p.dst = dst; p.ld_dst = ld_dst; p.dst_t = dst_t; p.ld_dst_t = ld_dst_t;
  p.amax = amax; p.flag = reinterpret_cast<int*>(flag); p.merge_amax = merge_amax;
  p.colsum = colsum_partial; p.telem_on_source = telem_on_source; p.tf32 = tf32;
  p.vec_src = aligned16(src, ld_src, es_src);
  p.vec_dst = aligned16(dst, ld_dst, es_dst);
  p.vec_dst_t = aligned16(dst_t, ld_dst_t, es_dst);
  const int st = cast_tma_try(src_dtype, dst_dtype, p, static_cast<cudaStream_t>(stream));
  if (st != APA_ERR_UNSUPPORTED) return st;
  return cast_dispatch(src_dtype, dst_dtype, p, static_cast<cudaStream_t>(stream));
}

extern "C" int apa_amax(const void* src, int dtype, int64_t n, float* amax, int32_t* flag, void* stream) {
  if ((!src && n > 0) || n < 0) return APA_ERR_INVALID;
  if (n == 0) return APA_OK;
  const int es = esize(dtype);
  if (!es) return APA_ERR_UNSUPPORTED;
  const int vec = (reinterpret_cast<uintptr_t>(src) & 15u) == 0;
  const int64_t work = (n * es + 15) / 16;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)num_sms() * 8));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* f = reinterpret_cast<int*>(flag);
  switch (dtype) {
    case APA_DT_F32: apa::launch_kernel(amax_kernel<APA_DT_F32>, dim3(grid), dim3(256), 0, s, 1, src, n, amax, f, vec); break;
    case APA_DT_F16: apa::launch_kernel(amax_kernel<APA_DT_F16>, dim3(grid), dim3(256), 0, s, 1, src, n, amax, f, vec); break;
    case APA_DT_BF16: apa::launch_kernel(amax_kernel<APA_DT_BF16>, dim3(grid), dim3(256), 0, s, 1, src, n, amax, f, vec); break;
    case APA_DT_E4M3: apa::launch_kernel(amax_kernel<APA_DT_E4M3>, dim3(grid), dim3(256), 0, s, 1, src, n, amax, f, vec); break;
    default: return APA_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

namespace apa {
namespace {
__global__ void merge_kernel(float* amax, int* flag, const float* src) {
  pdl_launch_dependents();
  pdl_wait();
  telem_commit(amax, flag, mag_bits(*src));
}
}  // namespace
}  // namespace apa

extern "C" int apa_merge_telemetry(float* amax, int32_t* flag, const float* src_amax, void* stream) {
  if (!src_amax) return APA_ERR_INVALID;
  apa::launch_kernel(apa::merge_kernel, dim3(1), dim3(1), 0, static_cast<cudaStream_t>(stream), 1, amax,
                     reinterpret_cast<int*>(flag), src_amax);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_underflow_ratio(const void* src, int dtype, int64_t n, float vmin, unsigned long long* counters,
                                   float* ratio_out, int running_max, void* stream) {
  if (n < 0 || (n > 0 && !src) || !counters || !ratio_out) return APA_ERR_INVALID;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 4));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case APA_DT_F32: apa::launch_kernel(underflow_kernel<APA_DT_F32>, dim3(grid), dim3(256), 0, s, 1, src, n, vmin, counters,
                                          ratio_out, running_max);
      break;
    case APA_DT_F16: apa::launch_kernel(underflow_kernel<APA_DT_F16>, dim3(grid), dim3(256), 0, s, 1, src, n, vmin, counters,
                                          ratio_out, running_max);
      break;
    case APA_DT_BF16: apa::launch_kernel(underflow_kernel<APA_DT_BF16>, dim3(grid), dim3(256), 0, s, 1, src, n, vmin, counters,
                                          ratio_out, running_max);
      break;
    case APA_DT_E4M3: apa::launch_kernel(underflow_kernel<APA_DT_E4M3>, dim3(grid), dim3(256), 0, s, 1, src, n, vmin, counters,
                                          ratio_out, running_max);
      break;
    default: return APA_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_colsum_finalize(const float* partial, int64_t nparts, int64_t cols, int work_dtype,
                                   float* out, int accumulate, void* stream) {
  if (!partial || !out || nparts < 0 || cols < 0) return APA_ERR_INVALID;
  if (cols == 0) return APA_OK;
  launch_colsum_finalize(partial, nparts, cols, work_dtype, out, accumulate, static_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_zero_list(int32_t* const* ptrs, int n, void* stream) {
  if (n < 0 || (n > 0 && !ptrs)) return APA_ERR_INVALID;
  if (n == 0) return APA_OK;
  apa::launch_kernel(apa::zero_list_kernel, dim3((n + 255) / 256), dim3(256), 0, static_cast<cudaStream_t>(stream), 1,
                     reinterpret_cast<int* const*>(ptrs), n);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_get_device_status(unsigned int* out, int clear) {
  if (!out) return APA_ERR_INVALID;
  if (cudaMemcpyFromSymbol(out, g_status, sizeof(unsigned int)) != cudaSuccess) return APA_ERR_CUDA;
  if (clear) {
    const unsigned int z = 0;
    if (cudaMemcpyToSymbol(g_status, &z, sizeof(z)) != cudaSuccess) return APA_ERR_CUDA;
  }
  return APA_OK;
}
