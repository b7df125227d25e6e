// K1, streaming version: cast + transposed copy + telemetry + bias partials
// with TMA in both directions.
//
// Same results as cast_kernel (every code, the telemetry pair, the per-64-row
// column partial sums) for the layouts the hot path uses: an fp32 / bf16 /
// fp16 source cast to E4M3, fp16 or fp32 (TF32-rounded at the TF32 rung),
// 16-byte aligned rows everywhere, with a row-major copy and/or a transposed
// copy. A persistent CTA per SM slot runs
//   warp 4      one thread streams 64 x 128 source tiles into a ring of
//               shared-memory stages with cp.async.bulk.tensor (128-byte
//               swizzle, zero fill past the edges), mbarrier full/empty pairs
//   warps 0..3  128 threads, each converting one 8 x 8 block of the tile in
//               registers: codes, a register transpose (byte / half-word
//               permutes), block max for telemetry, column sums for the bias
//               gradient; results go to swizzled staging tiles that one thread
//               writes out with TMA bulk-tensor stores (clipped at the edges).
// The thread -> block assignment (block row i = s, block column
// j = 8*(q%2) + (s + q/2)%8 for thread 8q + s), the per-thread order of the
// two 16-byte source chunks (fp32) and of the transposed rows make every
// shared-memory access of a quarter- or half-warp hit distinct banks for all
// source / destination type pairs.
#include <cuda.h>
#include <cmath>
#include <mutex>

#include "apa_common.cuh"

namespace apa {
namespace {

constexpr int kCTR = 64;            // source tile rows (= bias partial granularity)
constexpr int kCTC = 128;           // source tile columns
constexpr int kCastConsumers = 128;
constexpr int kCastTmaThreads = kCastConsumers + 32;
constexpr int kCastSmemBudget = 112 * 1024;   // two CTAs per SM

template <int SRC, int DST> struct TcCfg {
  static constexpr int ES = SRC == APA_DT_F32 ? 4 : 2;
  static constexpr int ED = DST == APA_DT_E4M3 ? 1 : DST == APA_DT_F16 ? 2 : 4;
  // fp32 destinations stage 64 KB per tile: one CTA per SM with a deeper ring
  static constexpr int kBudget = ED == 4 ? 200 * 1024 : kCastSmemBudget;
  static constexpr int kStageBytes = kCTR * kCTC * ES;         // 16 / 32 KB
  static constexpr int kBoxCols = 128 / ES;                    // 128-byte swizzle boxes
  static constexpr int kBoxes = kCTC / kBoxCols;
  static constexpr int kOutBytes = kCTR * kCTC * ED;           // one staging tile
  static constexpr int kCsumBytes = 8 * kCTC * 4;
  static constexpr int kFixed = 2 * kOutBytes + kCsumBytes + 128;
  static constexpr int kStagesFit = (kBudget - 1024 - kFixed) / kStageBytes;
  static constexpr int kStages = kStagesFit > 4 ? 4 : (kStagesFit < 1 ? 1 : kStagesFit);
  static constexpr int kSmemBytes = kStages * kStageBytes + kFixed + 1024;
};

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void cb_init(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(n) : "memory");
}
__device__ __forceinline__ void cb_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cb_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}
__device__ __forceinline__ bool cb_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait (2 s), status bit on expiry
__device__ __forceinline__ bool cb_wait(uint64_t* bar, uint32_t parity, unsigned int why) {
  if (cb_try(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!cb_try(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_status, why);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void ct_load(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          su32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void ct_store(const CUtensorMap* tm, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(su32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void ct_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void ct_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void ct_wait_all0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void ct_fence_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kCastConsumers) : "memory"); }
// consumer barrier that also returns the OR of every consumer's flag, so a
// timed-out wait in any thread ends the loop in all of them at the same tile
__device__ __forceinline__ bool consumers_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, 1, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(kCastConsumers)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// 4 x 4 byte transpose: in[k] holds row k (byte c = column c); out[c] holds
// column c (byte k = row k).
__device__ __forceinline__ void transpose4x4_b8(const uint32_t (&in)[4], uint32_t (&out)[4]) {
  const uint32_t x0 = prmt(in[0], in[1], 0x5140u), x1 = prmt(in[0], in[1], 0x7362u);
  const uint32_t x2 = prmt(in[2], in[3], 0x5140u), x3 = prmt(in[2], in[3], 0x7362u);
  out[0] = prmt(x0, x2, 0x5410u);
  out[1] = prmt(x0, x2, 0x7632u);
  out[2] = prmt(x1, x3, 0x5410u);
  out[3] = prmt(x1, x3, 0x7632u);
}

__device__ __forceinline__ bool f16x2_has_nan(uint32_t w) {
  return ((w & 0x7FFFu) > 0x7C00u) || (((w >> 16) & 0x7FFFu) > 0x7C00u);
}

struct TmaCastArgs {
  int64_t rows, cols;
  float* amax; int* flag;
  const float* merge_amax;
  float* colsum;
  int telem_on_source;
  int has_dst, has_dst_t;
  int tf32;                 // fp32 destination: stored values rounded to the TF32 grid
};

template <int SRC, int DST>
__global__ void __launch_bounds__(kCastTmaThreads, DST == APA_DT_F32 ? 1 : 2)
    cast_tma_kernel(const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmD,
                    const __grid_constant__ CUtensorMap tmT, TmaCastArgs p) {
  using C = TcCfg<SRC, DST>;
  constexpr int S = C::kStages;
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* sSrc = smem;                                   // S stages
  uint8_t* sOut = sSrc + S * C::kStageBytes;              // row-major staging (1024-aligned)
  uint8_t* sOutT = sOut + C::kOutBytes;                   // transposed staging
  float* sCsum = reinterpret_cast<float*>(sOutT + C::kOutBytes);   // [8][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(sCsum + 8 * kCTC);
  uint64_t* empty = full + S;
  __shared__ uint32_t red[kCastTmaThreads / 32];

  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int64_t tiles_r = (p.rows + kCTR - 1) / kCTR;
  const int64_t tiles_c = (p.cols + kCTC - 1) / kCTC;
  const int64_t ntiles = tiles_r * tiles_c;

  if (t == 0) {
    for (int s = 0; s < S; ++s) {
      cb_init(&full[s], 1);
      cb_init(&empty[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();   // the previous kernel's writes (the source, telemetry words) are visible

  uint32_t msrc = 0;
  if (warp == 4) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int64_t tr = tile / tiles_c, tc = tile - tr * tiles_c;
        if (!cb_wait(&empty[stage], phase ^ 1u, kStatusTimeoutEmpty)) { ok = false; break; }
        cb_expect_tx(&full[stage], C::kStageBytes);
#pragma unroll
        for (int b = 0; b < C::kBoxes; ++b)
          ct_load(sSrc + stage * C::kStageBytes + b * (kCTR * 128), &tmS, (int)(tc * kCTC + b * C::kBoxCols),
                  (int)(tr * kCTR), &full[stage]);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      // no TMA write may be in flight into this CTA's shared memory at exit
      for (int i = 0; ok && i < S; ++i) {
        if (!cb_wait(&empty[stage], phase ^ 1u, kStatusTimeoutEmpty)) ok = false;
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    const int q = t >> 3, s8 = t & 7;
    const int bi = s8;                                  // block row (8 source rows)
    const int bj = 8 * (q & 1) + ((s8 + (q >> 1)) & 7);  // block column (8 source columns)
    const int gflip = q & 1;                            // transposed-row order
    int stage = 0;
    uint32_t phase = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int64_t tr = tile / tiles_c, tc = tile - tr * tiles_c;
      // a failed (timed-out) wait still runs the arithmetic on whatever the
      // stage holds; barrier B below then ends the loop in every consumer
      const bool waited = cb_wait(&full[stage], phase, kStatusTimeoutFull);
      const uint8_t* st = sSrc + stage * C::kStageBytes;

      // ---- load the 8 x 8 block as fp32 ----
      float v[8][8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int R = 8 * bi + r;
        if constexpr (C::ES == 2) {
          const uint4 w = *reinterpret_cast<const uint4*>(st + (bj >> 3) * (kCTR * 128) + R * 128 +
                                                          ((((bj & 7) ^ r)) << 4));
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
          if constexpr (SRC == APA_DT_BF16) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              v[r][2 * k] = __uint_as_float(ws[k] << 16);
              v[r][2 * k + 1] = __uint_as_float(ws[k] & 0xFFFF0000u);
            }
          } else {
            const bool nan = f16x2_has_nan(ws[0]) || f16x2_has_nan(ws[1]) || f16x2_has_nan(ws[2]) ||
                             f16x2_has_nan(ws[3]);
            if (nan) {
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                v[r][2 * k] = f16_to_f32((uint16_t)(ws[k] & 0xFFFFu));
                v[r][2 * k + 1] = f16_to_f32((uint16_t)(ws[k] >> 16));
              }
            } else {
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                v[r][2 * k] = f16lo_to_f32(ws[k]);
                v[r][2 * k + 1] = f16hi_to_f32(ws[k]);
              }
            }
          }
        } else {
          const int f = (bj & 7) >> 2;   // which 16-byte half this thread reads first
          const uint8_t* rowp = st + (bj >> 2) * (kCTR * 128) + R * 128;
          const float4 a = *reinterpret_cast<const float4*>(rowp + (((2 * (bj & 3) + f) ^ r) << 4));
          const float4 b = *reinterpret_cast<const float4*>(rowp + (((2 * (bj & 3) + (f ^ 1)) ^ r) << 4));
          const float4 lo = f ? b : a, hi = f ? a : b;
          v[r][0] = lo.x; v[r][1] = lo.y; v[r][2] = lo.z; v[r][3] = lo.w;
          v[r][4] = hi.x; v[r][5] = hi.y; v[r][6] = hi.z; v[r][7] = hi.w;
        }
      }
      uint32_t m = 0;
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int c = 0; c < 8; ++c) m = max(m, mag_bits(v[r][c]));
      msrc = max(msrc, m);

      // ---- encode; code words per row: E4M3 2 words, fp16 4 words (fp32
      // values are stored from v, rounded to TF32 on the way out if asked) ----
      constexpr int W = C::ED == 4 ? 1 : C::ED * 2;
      uint32_t code[8][W];
      if constexpr (DST == APA_DT_F32) {
      } else if constexpr (DST == APA_DT_E4M3) {
        const bool big = m > kE4M3NaNThresholdBits;
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            uint32_t p01, p23;
            if (big) {
              p01 = e4m3x2_exact(v[r][4 * k], v[r][4 * k + 1]);
              p23 = e4m3x2_exact(v[r][4 * k + 2], v[r][4 * k + 3]);
            } else {
              p01 = e4m3x2_sat(v[r][4 * k], v[r][4 * k + 1]);
              p23 = e4m3x2_sat(v[r][4 * k + 2], v[r][4 * k + 3]);
            }
            code[r][k] = p01 | (p23 << 16);
          }
      } else {
        if (m > 0x7F800000u) {   // a NaN: keep sign and payload per element
#pragma unroll
          for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              code[r][k] = (uint32_t)f16_from_f32(v[r][2 * k]) | ((uint32_t)f16_from_f32(v[r][2 * k + 1]) << 16);
        } else {
#pragma unroll
          for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int k = 0; k < 4; ++k) code[r][k] = f16x2_from_f32(v[r][2 * k], v[r][2 * k + 1]);
        }
      }

      // ---- column sums of the cast values over the block's 8 rows ----
      float cs[8];
      if (p.colsum) {
#pragma unroll
        for (int c = 0; c < 8; ++c) cs[c] = 0.0f;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if constexpr (DST == APA_DT_F32) {
#pragma unroll
            for (int c = 0; c < 8; ++c) cs[c] += v[r][c];
          } else if constexpr (DST == APA_DT_E4M3) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t h = f16x2_from_e4m3x2((code[r][k >> 1] >> (16 * (k & 1))) & 0xFFFFu);
              cs[2 * k] += f16lo_to_f32(h);
              cs[2 * k + 1] += f16hi_to_f32(h);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              cs[2 * k] += f16lo_to_f32(code[r][k]);
              cs[2 * k + 1] += f16hi_to_f32(code[r][k]);
            }
          }
        }
      }

      // ---- E4M3 transposed block: T[c] = column c over rows 0..7 (the fp16
      // one is formed while it is written) ----
      uint32_t T[8][2];
      if constexpr (DST == APA_DT_E4M3) {
        if (p.has_dst_t) {
#pragma unroll
          for (int half = 0; half < 2; ++half)      // source columns 4*half .. +3
#pragma unroll
            for (int rg = 0; rg < 2; ++rg) {         // source rows 4*rg .. +3
              const uint32_t in[4] = {code[4 * rg][half], code[4 * rg + 1][half], code[4 * rg + 2][half],
                                      code[4 * rg + 3][half]};
              uint32_t out[4];
              transpose4x4_b8(in, out);
#pragma unroll
              for (int c = 0; c < 4; ++c) T[4 * half + c][rg] = out[c];
            }
        }
      }

      // the staging tiles of the previous tile must have been read by its stores
      if (t == 0) ct_wait_read0();
      // barrier B: stage fully read, staging free
      if (consumers_sync_or(!waited)) break;
      if (t == 0) cb_arrive(&empty[stage]);

      if (p.has_dst) {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int R = 8 * bi + r;
          if constexpr (DST == APA_DT_F32) {
            // two 16-byte chunks (columns 0-3, 4-7 of the block) in 32-column
            // boxes; the thread writes chunk f first (f = (j%8)/4)
            uint32_t w[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) w[c] = p.tf32 ? tf32_rn_bits(__float_as_uint(v[r][c])) : __float_as_uint(v[r][c]);
            const int f = (bj & 7) >> 2;
            uint8_t* rowp = sOut + (bj >> 2) * (kCTR * 128) + R * 128;
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const int k = kk ^ f;
              const uint4 val = k ? make_uint4(w[4], w[5], w[6], w[7]) : make_uint4(w[0], w[1], w[2], w[3]);
              *reinterpret_cast<uint4*>(rowp + (((2 * (bj & 3) + k) ^ r) << 4)) = val;
            }
          } else if constexpr (DST == APA_DT_E4M3) {
            *reinterpret_cast<uint2*>(sOut + R * 128 + (((bj >> 1) ^ r) << 4) + ((bj & 1) << 3)) =
                make_uint2(code[r][0], code[r][1]);
          } else {
            *reinterpret_cast<uint4*>(sOut + (bj >> 3) * (kCTR * 128) + R * 128 + (((bj & 7) ^ r) << 4)) =
                make_uint4(code[r][0], code[r][1], code[r][2], code[r][3]);
          }
        }
      }
      if (p.has_dst_t) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int cc = c ^ gflip;
          const int R = 8 * bj + cc;
          if constexpr (DST == APA_DT_F32) {
            // column cc over the block's 8 rows: chunks rows 0-3 / 4-7 in the
            // 32-row boxes of the transposed tile; chunk i/4 first
            uint32_t w[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float e = gflip ? v[k][c ^ 1] : v[k][c];
              w[k] = p.tf32 ? tf32_rn_bits(__float_as_uint(e)) : __float_as_uint(e);
            }
            const int f = bi >> 2;
            uint8_t* rowp = sOutT + (bi >> 2) * (kCTC * 128) + R * 128;
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              const int k = kk ^ f;
              const uint4 val = k ? make_uint4(w[4], w[5], w[6], w[7]) : make_uint4(w[0], w[1], w[2], w[3]);
              *reinterpret_cast<uint4*>(rowp + (((2 * (bi & 3) + k) ^ (R & 7)) << 4)) = val;
            }
          } else if constexpr (DST == APA_DT_E4M3) {
            const uint32_t w0 = gflip ? T[c ^ 1][0] : T[c][0];
            const uint32_t w1 = gflip ? T[c ^ 1][1] : T[c][1];
            *reinterpret_cast<uint2*>(sOutT + R * 64 + (((bi >> 1) ^ ((R >> 1) & 3)) << 4) + ((bi & 1) << 3)) =
                make_uint2(w0, w1);
          } else {
            // halves of rows 2k, 2k+1 at column cc (cc and c share the word c/2)
            const uint32_t sel = (cc & 1) ? 0x7632u : 0x5410u;
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) w[k] = prmt(code[2 * k][c >> 1], code[2 * k + 1][c >> 1], sel);
            *reinterpret_cast<uint4*>(sOutT + R * 128 + ((bi ^ (R & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (p.colsum) {
        float4* cp = reinterpret_cast<float4*>(sCsum + bi * kCTC + 8 * bj);
        cp[0] = make_float4(cs[0], cs[1], cs[2], cs[3]);
        cp[1] = make_float4(cs[4], cs[5], cs[6], cs[7]);
      }
      ct_fence_smem();
      consumers_sync();                                  // barrier A: staging complete
      if (t == 0) {
        const int x = (int)(tc * kCTC), y = (int)(tr * kCTR);
        if (p.has_dst) {
          if constexpr (DST == APA_DT_E4M3) {
            ct_store(&tmD, sOut, x, y);
          } else if constexpr (DST == APA_DT_F16) {
            ct_store(&tmD, sOut, x, y);
            if (x + 64 < p.cols) ct_store(&tmD, sOut + kCTR * 128, x + 64, y);
          } else {
#pragma unroll
            for (int b = 0; b < 4; ++b)
              if (x + 32 * b < p.cols) ct_store(&tmD, sOut + b * (kCTR * 128), x + 32 * b, y);
          }
        }
        if (p.has_dst_t) {
          if constexpr (DST == APA_DT_F32) {
            ct_store(&tmT, sOutT, y, x);
            if (y + 32 < p.rows) ct_store(&tmT, sOutT + kCTC * 128, y + 32, x);
          } else {
            ct_store(&tmT, sOutT, y, x);
          }
        }
        ct_commit();
      }
      if (p.colsum) {
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) sum += sCsum[i * kCTC + t];
        const int64_t col = tc * kCTC + t;
        if (col < p.cols) p.colsum[tr * p.cols + col] = sum;
      }
      if (++stage == S) { stage = 0; phase ^= 1u; }
    }
    if (t == 0) ct_wait_all0();
  }

  // telemetry: the cast values' max is the cast of the source max
  uint32_t mag = msrc;
  if (!p.telem_on_source) {
    if constexpr (DST == APA_DT_E4M3) mag = e4m3_mag_bits(e4m3_from_f32(__uint_as_float(msrc)));
    else if constexpr (DST == APA_DT_F16) mag = mag_bits(f16_to_f32(f16_from_f32(__uint_as_float(msrc))));
  }
  mag = warp_max_u32(mag);
  if (lane == 0) red[warp] = mag;
  __syncthreads();
  if (t < 32) {
    uint32_t mm = t < kCastTmaThreads / 32 ? red[t] : 0u;
    mm = warp_max_u32(mm);
    if (t == 0) {
      telem_commit(p.amax, p.flag, mm);
      if (blockIdx.x == 0 && p.merge_amax) telem_commit(p.amax, p.flag, mag_bits(*p.merge_amax));
    }
  }
}

// dims {inner, outer}, row pitch in bytes, box {bx, by}
bool cast_map(CUtensorMap* tm, CUtensorMapDataType dt, const void* ptr, int64_t inner, int64_t outer,
              int64_t pitch_bytes, int bx, int by, CUtensorMapSwizzle sw) {
  gemm::EncodeFn enc = gemm::get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)pitch_bytes};
  cuuint32_t box[2] = {(cuuint32_t)bx, (cuuint32_t)by};
  cuuint32_t estr[2] = {1, 1};
  return enc(tm, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


template <int SRC, int DST>
int launch_cast_tma_t(const CastParams& cp, cudaStream_t s) {
  using C = TcCfg<SRC, DST>;
  static std::once_flag once;
  static int blocks_per_sm = 0;
  std::call_once(once, [] {
    if (cudaFuncSetAttribute(cast_tma_kernel<SRC, DST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemBytes) != cudaSuccess)
      return;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, cast_tma_kernel<SRC, DST>, kCastTmaThreads,
                                                      C::kSmemBytes) == cudaSuccess)
      blocks_per_sm = n;
  });
  if (blocks_per_sm < 1) {
    (void)cudaGetLastError();
    return APA_ERR_UNSUPPORTED;
  }
  const CUtensorMapDataType sdt = SRC == APA_DT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : SRC == APA_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUtensorMapDataType ddt = DST == APA_DT_E4M3  ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                  : DST == APA_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap ms, md, mt;
  if (!cast_map(&ms, sdt, cp.src, cp.cols, cp.rows, cp.ld_src * C::ES, C::kBoxCols, kCTR,
                CU_TENSOR_MAP_SWIZZLE_128B))
    return APA_ERR_UNSUPPORTED;
  md = ms;
  mt = ms;
  if (cp.dst) {
    const int bx = 128 / C::ED;
    if (!cast_map(&md, ddt, cp.dst, cp.cols, cp.rows, cp.ld_dst * C::ED, bx, kCTR, CU_TENSOR_MAP_SWIZZLE_128B))
      return APA_ERR_UNSUPPORTED;
  }
  if (cp.dst_t) {
    const CUtensorMapSwizzle sw = DST == APA_DT_E4M3 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    const int bx = DST == APA_DT_F32 ? 32 : kCTR;
    if (!cast_map(&mt, ddt, cp.dst_t, cp.rows, cp.cols, cp.ld_dst_t * C::ED, bx, kCTC, sw))
      return APA_ERR_UNSUPPORTED;
  }
  TmaCastArgs a;
  a.rows = cp.rows; a.cols = cp.cols;
  a.amax = cp.amax; a.flag = cp.flag; a.merge_amax = cp.merge_amax;
  a.colsum = cp.colsum; a.telem_on_source = cp.telem_on_source;
  a.has_dst = cp.dst != nullptr; a.has_dst_t = cp.dst_t != nullptr;
  a.tf32 = cp.tf32;
  const int64_t tiles = ((cp.rows + kCTR - 1) / kCTR) * ((cp.cols + kCTC - 1) / kCTC);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)num_sms() * blocks_per_sm));
  if (launch_kernel(cast_tma_kernel<SRC, DST>, dim3((unsigned)grid), dim3(kCastTmaThreads), C::kSmemBytes, s, 1, ms,
                    md, mt, a) != cudaSuccess)
    return APA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

bool tma_ok(const void* p, int64_t ld, int es) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && ((ld * es) & 15) == 0;
}

}  // namespace

// The streaming kernel when it applies (E4M3 / fp16 / fp32 destination, at least one
// output copy, 16-byte aligned rows, sizes a tensor map can describe);
// APA_ERR_UNSUPPORTED otherwise, and the caller uses cast_kernel.
int cast_tma_try(int src_dt, int dst_dt, const CastParams& p, cudaStream_t s) {
  if (dst_dt != APA_DT_E4M3 && dst_dt != APA_DT_F16 && dst_dt != APA_DT_F32) return APA_ERR_UNSUPPORTED;
  if (src_dt != APA_DT_F32 && src_dt != APA_DT_BF16 && src_dt != APA_DT_F16) return APA_ERR_UNSUPPORTED;
  if (!p.dst && !p.dst_t) return APA_ERR_UNSUPPORTED;
  if (p.rows <= 0 || p.cols <= 0 || p.rows >= (1ll << 31) || p.cols >= (1ll << 31)) return APA_ERR_UNSUPPORTED;
  const int es = src_dt == APA_DT_F32 ? 4 : 2, ed = dst_dt == APA_DT_E4M3 ? 1 : dst_dt == APA_DT_F16 ? 2 : 4;
  if (!tma_ok(p.src, p.ld_src, es)) return APA_ERR_UNSUPPORTED;
  if (p.dst && !tma_ok(p.dst, p.ld_dst, ed)) return APA_ERR_UNSUPPORTED;
  if (p.dst_t && !tma_ok(p.dst_t, p.ld_dst_t, ed)) return APA_ERR_UNSUPPORTED;
#define APA_TC(S_, D_) \
  if (src_dt == S_ && dst_dt == D_) return launch_cast_tma_t<S_, D_>(p, s);
  APA_TC(APA_DT_F32, APA_DT_E4M3)
  APA_TC(APA_DT_BF16, APA_DT_E4M3)
  APA_TC(APA_DT_F16, APA_DT_E4M3)
  APA_TC(APA_DT_F32, APA_DT_F16)
  APA_TC(APA_DT_BF16, APA_DT_F16)
  APA_TC(APA_DT_F16, APA_DT_F16)
  APA_TC(APA_DT_F32, APA_DT_F32)
  APA_TC(APA_DT_BF16, APA_DT_F32)
  APA_TC(APA_DT_F16, APA_DT_F32)
#undef APA_TC
  return APA_ERR_UNSUPPORTED;
}

}  // namespace apa
