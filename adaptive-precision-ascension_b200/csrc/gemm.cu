// K2/K3/K4: tcgen05 GEMMs for the three ladder rungs with fused epilogues.
//
// D[M,N] = A[M,K] . B[N,K]^T with both operands K-major (row-major with the
// reduction dimension contiguous), fp32 accumulation in tensor memory.
//
//   rung FP8  -> tcgen05.mma kind::f8f6f4 (E4M3 x E4M3)
//   rung FP16 -> tcgen05.mma kind::f16    (F16 x F16)
//   rung TF32 -> tcgen05.mma kind::tf32   (fp32 storage, TF32 multiply)
//
// One CTA per SM, persistent over output tiles of 128 x BN:
//   warp 0      one thread issues TMA loads (128-byte swizzle) into a
//               kStages-deep shared-memory ring (mbarrier full/empty pairs)
//   warp 1      allocates 2*BN TMEM columns; one thread issues tcgen05.mma
//               (4 per 128-byte K slab) and tcgen05.commit to release stages
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, apply
//               the op's epilogue, store to global; the accumulator is double
//               buffered so the epilogue of tile i overlaps the MMAs of i+1.
//
// Epilogues (the reference's work after each GEMM, fused so no extra pass
// reads the output back from HBM):
//   FWD    y = acc + bias (layers.py:164-182), fp32 out (FP8, TF32) or fp16
//          out (FP16); amax/NaN telemetry of y (layers.py:186).
//   DGRAD  dx = cast(cast(acc, working dtype), x dtype): the autograd engine's
//          re-cast to x_cast's dtype followed by ToCopyBackward; the
//          boundary_cast backward-hook telemetry (manager.py:79-84) is taken
//          on the working-dtype value.
//   WGRAD  nonzero/underflow counts of the fp32 (FP16: fp16-rounded) weight
//          gradient (telemetry.py:23-39), then master.grad =
//          f32(cast(acc, working dtype)) (layers.py:277-282 + the engine's
//          re-cast + manager.py:191-204). The last CTA to finish turns the
//          counts into the ratio and folds it into gpu_underflow_ratio
//          (layers.py:404-407) without a host round trip.
//
// Every mbarrier wait is bounded (2 s); on expiry the kernel sets a bit in
// the library status word and unwinds instead of spinning forever.
#include <cuda.h>
#include <mutex>
#include "apa_common.cuh"

namespace apa {
int num_sms();
namespace gemm {

constexpr int BM = 128;
constexpr int kSlab = 128;            // K bytes per pipeline stage (one swizzle row)
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;

enum { KIND_E4M3 = 0, KIND_F16 = 1, KIND_TF32 = 2 };
enum { EPI_FWD = 0, EPI_DGRAD = 1, EPI_WGRAD = 2 };

template <int KIND> struct KindInfo;
template <> struct KindInfo<KIND_E4M3> { static constexpr int bytes = 1; static constexpr uint32_t fmt = 0; };
template <> struct KindInfo<KIND_F16> { static constexpr int bytes = 2; static constexpr uint32_t fmt = 0; };
template <> struct KindInfo<KIND_TF32> { static constexpr int bytes = 4; static constexpr uint32_t fmt = 2; };

template <int BN> struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = BM * kSlab;
  static constexpr int kBBytes = BN * kSlab;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;
};

struct EpiArgs {
  void* out; int64_t ldo; int out_dt; int vec_out;
  const void* bias;                 // FWD: working-dtype bias (nullable)
  float* amax; int* flag;           // FWD: module telemetry; DGRAD: boundary_cast telemetry
  unsigned long long* counters;     // WGRAD: [nonzero, underflow, ticket], zero on entry
  float* ratio_max;                 // WGRAD: module gpu_underflow_ratio
  float vmin;                       // WGRAD: underflow threshold as fp32
  int accumulate;                   // WGRAD: add into out instead of overwriting
  int M, N, K;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int why) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_status, why);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms
// stacked at a 1024-byte stride. Advancing along K inside the 128-byte row is
// done by adding the byte offset to the start address.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: fp32 accumulator, A/B formats, both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24.
template <int KIND, int BN>
__host__ __device__ constexpr uint32_t idesc() {
  return (1u << 4) | (KindInfo<KIND>::fmt << 7) | (KindInfo<KIND>::fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

template <int KIND>
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
  if constexpr (KIND == KIND_E4M3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(accumulate));
  } else if constexpr (KIND == KIND_F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(accumulate));
  }
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Epilogue helpers
// ---------------------------------------------------------------------------
template <int KIND>
__device__ __forceinline__ float bias_value(const void* bias, int n) {
  if constexpr (KIND == KIND_E4M3) return e4m3_to_f32(static_cast<const uint8_t*>(bias)[n]);
  else if constexpr (KIND == KIND_F16) return f16_to_f32(static_cast<const uint16_t*>(bias)[n]);
  else return static_cast<const float*>(bias)[n];
}

// Write 32 fp32 values (as bits) of one row; cnt valid columns.
__device__ __forceinline__ void store_row(const EpiArgs& ea, int row, int col0, int cnt, const uint32_t (&w)[32],
                                          int out_dt) {
  if (out_dt == APA_DT_F32) {
    float* o = static_cast<float*>(ea.out) + (int64_t)row * ea.ldo + col0;
    if (cnt == 32 && ea.vec_out) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<uint4*>(o)[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < cnt) o[j] = __uint_as_float(w[j]);
    }
  } else {
    // 16-bit outputs: w holds the 16-bit codes
    uint16_t* o = static_cast<uint16_t*>(ea.out) + (int64_t)row * ea.ldo + col0;
    if (cnt == 32 && ea.vec_out) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<uint4*>(o)[q] =
            make_uint4(w[8 * q] | (w[8 * q + 1] << 16), w[8 * q + 2] | (w[8 * q + 3] << 16),
                       w[8 * q + 4] | (w[8 * q + 5] << 16), w[8 * q + 6] | (w[8 * q + 7] << 16));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < cnt) o[j] = (uint16_t)w[j];
    }
  }
}

struct EpiState {
  uint32_t mag = 0;
  uint32_t nz = 0, uf = 0;
};

template <int KIND, int EPI>
__device__ __forceinline__ void epilogue_chunk(const EpiArgs& ea, int row, int col0, uint32_t (&r)[32],
                                               EpiState& st) {
  const int cnt = min(32, ea.N - col0);
  if constexpr (EPI == EPI_FWD) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float v = __uint_as_float(r[j]);
      if (ea.bias != nullptr && j < cnt) v += bias_value<KIND>(ea.bias, col0 + j);
      if constexpr (KIND == KIND_F16) {
        const uint16_t h = f16_from_f32(v);
        if (j < cnt) st.mag = max(st.mag, mag_bits(f16_to_f32(h)));
        r[j] = h;
      } else {
        if (j < cnt) st.mag = max(st.mag, mag_bits(v));
        r[j] = __float_as_uint(v);
      }
    }
    store_row(ea, row, col0, cnt, r, KIND == KIND_F16 ? APA_DT_F16 : APA_DT_F32);
  } else if constexpr (EPI == EPI_DGRAD) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float v = __uint_as_float(r[j]);
      float qv;          // value after the re-cast to the working dtype
      uint32_t outc;     // code in the output dtype
      if constexpr (KIND == KIND_E4M3) {
        const uint32_t c = e4m3_from_f32(v);
        qv = e4m3_to_f32(c);
        if (j < cnt) st.mag = max(st.mag, e4m3_mag_bits(c));
        outc = ea.out_dt == APA_DT_F16 ? (uint32_t)e4m3_to_f16(c)
               : ea.out_dt == APA_DT_BF16 ? (__float_as_uint(qv) >> 16)   // exact: 3 mantissa bits
                                          : __float_as_uint(qv);
      } else if constexpr (KIND == KIND_F16) {
        const uint16_t h = f16_from_f32(v);
        qv = f16_to_f32(h);
        if (j < cnt) st.mag = max(st.mag, mag_bits(qv));
        outc = ea.out_dt == APA_DT_F16 ? (uint32_t)h
               : ea.out_dt == APA_DT_BF16 ? (uint32_t)bf16_from_f32(qv)
                                          : __float_as_uint(qv);
      } else {
        qv = v;
        if (j < cnt) st.mag = max(st.mag, mag_bits(qv));
        outc = ea.out_dt == APA_DT_F16 ? (uint32_t)f16_from_f32(qv)
               : ea.out_dt == APA_DT_BF16 ? (uint32_t)bf16_from_f32(qv)
                                          : __float_as_uint(qv);
      }
      r[j] = outc;
    }
    store_row(ea, row, col0, cnt, r, ea.out_dt);
  } else {
    const uint32_t vmin_bits = __float_as_uint(ea.vmin);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float v = __uint_as_float(r[j]);
      if constexpr (KIND == KIND_F16) v = f16_to_f32(f16_from_f32(v));   // the fp16 GEMM output
      if constexpr (KIND != KIND_TF32) {
        // |v| > 0 and |v| < vmin, compared as magnitudes (NaN is neither)
        const uint32_t m = mag_bits(v);
        const bool nonzero = m != 0u && m <= 0x7F800000u;
        if (j < cnt) {
          st.nz += nonzero ? 1u : 0u;
          st.uf += (nonzero && m < vmin_bits) ? 1u : 0u;
        }
      }
      float q;
      if constexpr (KIND == KIND_E4M3) q = e4m3_to_f32(e4m3_from_f32(v));
      else q = v;
      r[j] = __float_as_uint(q);
    }
    if (ea.accumulate) {
      const float* o = static_cast<const float*>(ea.out) + (int64_t)row * ea.ldo + col0;
      for (int j = 0; j < cnt; ++j) r[j] = __float_as_uint(o[j] + __uint_as_float(r[j]));
    }
    store_row(ea, row, col0, cnt, r, APA_DT_F32);
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int KIND, int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, EpiArgs ea) {
  using C = Cfg<BN>;
  constexpr int kStages = C::kStages;
  constexpr int kElemPerSlab = kSlab / KindInfo<KIND>::bytes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smA = smem;
  uint8_t* smB = smem + kStages * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * C::kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = (ea.N + BN - 1) / BN;
  const int num_tiles = ((ea.M + BM - 1) / BM) * num_n;
  const int kb_count = (int)(((int64_t)ea.K * KindInfo<KIND>::bytes + kSlab - 1) / kSlab);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiThreads);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m_blk = tile / num_n, n_blk = tile - (tile / num_n) * num_n;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kStatusTimeoutEmpty)) { ok = false; break; }
          mbar_expect_tx(&full[stage], C::kStageBytes);
          tma_load_2d(smA + stage * C::kABytes, &tmA, kb * kElemPerSlab, m_blk * BM, &full[stage]);
          tma_load_2d(smB + stage * C::kBBytes, &tmB, kb * kElemPerSlab, n_blk * BN, &full[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      // producer tail: wait until the MMAs have released every stage, so no
      // tensor-core read of shared memory is outstanding when the CTA exits
      for (int i = 0; ok && i < kStages; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, kStatusTimeoutEmpty)) ok = false;
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      constexpr uint32_t id = idesc<KIND, BN>();
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
        if (!mbar_wait(&tempty[acc], acc_par ^ 1u, kStatusTimeoutAcc)) { ok = false; break; }
        fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&full[stage], phase, kStatusTimeoutFull)) { ok = false; break; }
          fence_after();
          const uint32_t a0 = smem_u32(smA + stage * C::kABytes);
          const uint32_t b0 = smem_u32(smB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < kSlab / 32; ++k)
            mma<KIND>(d, sdesc(a0 + 32 * k), sdesc(b0 + 32 * k), id, (kb | k) != 0 ? 1u : 0u);
          mma_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit(&tfull[acc]);
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5 -> TMEM lane quarters 2,3,0,1
    const int q = warp & 3;
    EpiState st;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
      if (!mbar_wait(&tfull[acc], acc_par, kStatusTimeoutAcc)) break;
      fence_after();
      const int m_blk = tile / num_n, n_blk = tile - (tile / num_n) * num_n;
      const int row = m_blk * BM + q * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        const int col0 = n_blk * BN + c;
        if (col0 >= ea.N) break;   // warp-uniform
        uint32_t r[32];
        tmem_ld32(tbase + (uint32_t)c, r);
        if (row < ea.M) epilogue_chunk<KIND, EPI>(ea, row, col0, r, st);
      }
      fence_before();
      mbar_arrive(&tempty[acc]);
    }
    // per-warp telemetry commit
    if constexpr (EPI == EPI_WGRAD) {
      uint32_t nz = st.nz, uf = st.uf;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        nz += __shfl_xor_sync(0xFFFFFFFFu, nz, o);
        uf += __shfl_xor_sync(0xFFFFFFFFu, uf, o);
      }
      if (lane == 0 && ea.counters) {
        if (nz) atomicAdd(&ea.counters[0], (unsigned long long)nz);
        if (uf) atomicAdd(&ea.counters[1], (unsigned long long)uf);
      }
    } else {
      const uint32_t m = warp_max_u32(st.mag);
      if (lane == 0) telem_commit(ea.amax, ea.flag, m);
    }
    if constexpr (EPI == EPI_WGRAD) {
      // named barrier over the 4 epilogue warps, then one ticket per CTA
      asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory");
      if (threadIdx.x == 64 && ea.counters) {
        __threadfence();
        const unsigned long long ticket = atomicAdd(&ea.counters[2], 1ull);
        if (ticket == (unsigned long long)gridDim.x - 1ull) {
          __threadfence();
          const unsigned long long nzc = atomicAdd(&ea.counters[0], 0ull);
          const unsigned long long ufc = atomicAdd(&ea.counters[1], 0ull);
          float ratio = 0.0f;
          if (nzc != 0ull) ratio = __fdiv_rn(__ull2float_rn(ufc), __ull2float_rn(nzc));
          if (ea.ratio_max) {
            const float old = *ea.ratio_max;
            *ea.ratio_max = (old != old) ? old : fmaxf(old, ratio);
          }
          ea.counters[0] = 0ull;
          ea.counters[1] = 0ull;
          ea.counters[2] = 0ull;
        }
      }
    }
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"((uint32_t)C::kTmemCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// 2-D K-major operand: dims {K (inner), rows}, row pitch ld elements,
// box {128 bytes of K, box_rows rows}, 128-byte swizzle, zero fill out of bounds.
int make_map(CUtensorMap* tm, int kind, const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  EncodeFn enc = get_encode();
  if (!enc) return APA_ERR_CUDA;
  const int es = kind == KIND_E4M3 ? 1 : kind == KIND_F16 ? 2 : 4;
  const CUtensorMapDataType dt = kind == KIND_E4M3  ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : kind == KIND_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0 || ((ld * es) & 15) != 0) return APA_ERR_ALIGN;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {(cuuint32_t)(kSlab / es), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? APA_OK : APA_ERR_CUDA;
}

template <int KIND, int BN, int EPI>
int launch_t(const void* A, int64_t lda, const void* B, int64_t ldb, EpiArgs ea, int grid_cap, cudaStream_t s) {
  using C = Cfg<BN>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(gemm_kernel<KIND, BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return APA_ERR_CUDA;
  CUtensorMap ta, tb;
  int st = make_map(&ta, KIND, A, ea.M, ea.K, lda, BM);
  if (st) return st;
  st = make_map(&tb, KIND, B, ea.N, ea.K, ldb, BN);
  if (st) return st;
  const int tiles = ((ea.M + BM - 1) / BM) * ((ea.N + BN - 1) / BN);
  int grid = std::min(tiles, grid_cap > 0 ? grid_cap : num_sms());
  if (grid < 1) grid = 1;
  gemm_kernel<KIND, BN, EPI><<<grid, kThreads, C::kSmemBytes, s>>>(ta, tb, ea);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

template <int KIND, int EPI>
int launch_bn(const void* A, int64_t lda, const void* B, int64_t ldb, EpiArgs ea, int bn, int grid_cap,
              cudaStream_t s) {
  if (bn == 256) return launch_t<KIND, 256, EPI>(A, lda, B, ldb, ea, grid_cap, s);
  return launch_t<KIND, 128, EPI>(A, lda, B, ldb, ea, grid_cap, s);
}

}  // namespace gemm

// Choose the N tile: 256 keeps shared-memory traffic per MMA lowest; 128 when
// N is small or 256-wide tiles would leave SMs idle.
int pick_bn(int64_t M, int64_t N) {
  if (N <= 128) return 128;
  const int64_t t256 = ((M + 127) / 128) * ((N + 255) / 256);
  if (t256 >= num_sms()) return 256;
  const int64_t t128 = ((M + 127) / 128) * ((N + 127) / 128);
  return t128 > t256 ? 128 : 256;
}

int gemm_dispatch(int rung, int epi, const void* A, int64_t lda, const void* B, int64_t ldb, gemm::EpiArgs ea,
                  int bn, int grid_cap, cudaStream_t s) {
  using namespace gemm;
  if (bn != 128 && bn != 256) bn = pick_bn(ea.M, ea.N);
#define APA_EPI_CASE(KIND)                                                               \
  switch (epi) {                                                                          \
    case EPI_FWD: return launch_bn<KIND, EPI_FWD>(A, lda, B, ldb, ea, bn, grid_cap, s);   \
    case EPI_DGRAD: return launch_bn<KIND, EPI_DGRAD>(A, lda, B, ldb, ea, bn, grid_cap, s); \
    case EPI_WGRAD: return launch_bn<KIND, EPI_WGRAD>(A, lda, B, ldb, ea, bn, grid_cap, s); \
    default: return APA_ERR_INVALID;                                                      \
  }
  switch (rung) {
    case APA_RUNG_FP8: APA_EPI_CASE(KIND_E4M3)
    case APA_RUNG_FP16: APA_EPI_CASE(KIND_F16)
    case APA_RUNG_TF32: APA_EPI_CASE(KIND_TF32)
    default: return APA_ERR_INVALID;
  }
#undef APA_EPI_CASE
}

}  // namespace apa

using apa::gemm::EpiArgs;

namespace {

int check_dims(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return APA_ERR_INVALID;
  if (M > (1ll << 31) - 256 || N > (1ll << 31) - 256 || K > (1ll << 31) - 256) return APA_ERR_INVALID;
  return APA_OK;
}

EpiArgs blank(int64_t M, int64_t N, int64_t K) {
  EpiArgs ea;
  ea.out = nullptr; ea.ldo = 0; ea.out_dt = APA_DT_F32; ea.vec_out = 0;
  ea.bias = nullptr; ea.amax = nullptr; ea.flag = nullptr;
  ea.counters = nullptr; ea.ratio_max = nullptr; ea.vmin = 0.0f; ea.accumulate = 0;
  ea.M = (int)M; ea.N = (int)N; ea.K = (int)K;
  return ea;
}

int out_vec(const void* p, int64_t ld, int es) {
  return ((reinterpret_cast<uintptr_t>(p) & 15u) == 0 && ((ld * es) & 15) == 0) ? 1 : 0;
}

}  // namespace

extern "C" int apa_linear_fwd(int rung, const void* xq, int64_t ldx, const void* wq, int64_t ldw, const void* bias_q,
                              void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, float* amax, int32_t* flag,
                              void* stream) {
  if (int st = check_dims(M, N, K)) return st;
  if (!xq || !wq || !y || ldy < N || ldx < K || ldw < K) return APA_ERR_INVALID;
  EpiArgs ea = blank(M, N, K);
  ea.out = y; ea.ldo = ldy;
  ea.out_dt = rung == APA_RUNG_FP16 ? APA_DT_F16 : APA_DT_F32;
  ea.vec_out = out_vec(y, ldy, rung == APA_RUNG_FP16 ? 2 : 4);
  ea.bias = bias_q; ea.amax = amax; ea.flag = reinterpret_cast<int*>(flag);
  return apa::gemm_dispatch(rung, apa::gemm::EPI_FWD, xq, ldx, wq, ldw, ea, 0, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int apa_linear_dgrad(int rung, const void* dyq, int64_t lddy, const void* wqt, int64_t ldwt, void* dx,
                                int dx_dtype, int64_t lddx, int64_t M, int64_t N, int64_t K, float* bc_amax,
                                int32_t* bc_flag, void* stream) {
  // dx[M, K] = dyq[M, N] . wq[N, K]; the GEMM reduces over N.
  if (int st = check_dims(M, K, N)) return st;
  if (!dyq || !wqt || !dx || lddx < K || lddy < N || ldwt < N) return APA_ERR_INVALID;
  if (dx_dtype != APA_DT_F32 && dx_dtype != APA_DT_BF16 && dx_dtype != APA_DT_F16) return APA_ERR_UNSUPPORTED;
  EpiArgs ea = blank(M, K, N);
  ea.out = dx; ea.ldo = lddx; ea.out_dt = dx_dtype;
  ea.vec_out = out_vec(dx, lddx, dx_dtype == APA_DT_F32 ? 4 : 2);
  ea.amax = bc_amax; ea.flag = reinterpret_cast<int*>(bc_flag);
  return apa::gemm_dispatch(rung, apa::gemm::EPI_DGRAD, dyq, lddy, wqt, ldwt, ea, 0, 0,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int apa_linear_wgrad(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt, float* dw,
                                int64_t lddw, int64_t M, int64_t N, int64_t K, int accumulate,
                                unsigned long long* counters, float* ratio_max, void* stream) {
  // dw[N, K] = dyq[M, N]^T . xq[M, K]; operands are the transposed copies
  // dyqt[N, M] and xqt[K, M]; the GEMM reduces over M.
  if (int st = check_dims(N, K, M)) return st;
  if (!dyqt || !xqt || !dw || lddw < K || lddyt < M || ldxt < M) return APA_ERR_INVALID;
  if (rung != APA_RUNG_TF32 && !counters) return APA_ERR_INVALID;
  EpiArgs ea = blank(N, K, M);
  ea.out = dw; ea.ldo = lddw; ea.out_dt = APA_DT_F32; ea.vec_out = out_vec(dw, lddw, 4);
  ea.accumulate = accumulate; ea.counters = counters; ea.ratio_max = ratio_max;
  ea.vmin = rung == APA_RUNG_FP8 ? 0.015625f : rung == APA_RUNG_FP16 ? 6.1035e-5f : 0.0f;
  return apa::gemm_dispatch(rung, apa::gemm::EPI_WGRAD, dyqt, lddyt, xqt, ldxt, ea, 0, 0,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int apa_gemm_tn(int rung, int epilogue, const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                           int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, int tile_n, int grid_cap,
                           void* stream) {
  // Plain D = A . B^T with the epilogue of the given op and no telemetry
  // side effects; used to time the bare GEMM against the fused versions.
  if (int st = check_dims(M, N, K)) return st;
  if (!A || !B || !out) return APA_ERR_INVALID;
  EpiArgs ea = blank(M, N, K);
  ea.out = out; ea.ldo = ldo; ea.out_dt = out_dtype;
  ea.vec_out = out_vec(out, ldo, out_dtype == APA_DT_F32 ? 4 : 2);
  return apa::gemm_dispatch(rung, epilogue, A, lda, B, ldb, ea, tile_n, grid_cap, static_cast<cudaStream_t>(stream));
}
