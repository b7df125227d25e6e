// AdamW on an fp32 master weight fused with the next step's working copy.
//
// The reference updates the masters with torch.optim.AdamW and re-casts them
// at the next pre_step (manager.py:145-172, layers.py:368-372): the update
// reads p, g, m, v and writes p, m, v, and the refresh reads p once more to
// write W_q and W_q^T. Here one pass does both, with every global access a
// bulk transfer:
//   warp 16     one thread streams 32 x 64 tiles of p, g, m, v (two 32-column
//               boxes each, 128-byte swizzle, zero fill past the edges) into a
//               ring of shared-memory stages
//   warps 0..15 512 threads; thread (w, lane) owns row `lane` and the four
//               columns 4w..4w+3 of the tile (box w/8, 16-byte chunk w%8,
//               conflict-free under the swizzle). It updates the four
//               elements in place in the stage (torch.optim.AdamW order of
//               operations), keeps the new p in registers, casts them, and
//               writes the row-major working copy (swizzled) and the
//               transposed copy (dense, one element per lane of a 32-element
//               row) into staging tiles. The IEEE divisions and square root
//               make one element a long dependent chain: sixteen warps keep
//               the SM issuing while the chains wait.
// One thread then stores p, m, v straight from the stage and both copies from
// staging with TMA bulk-tensor stores (clipped at the edges). A stage is handed
// back to the producer one tile later, once its stores have read it.
//
// The working copies and the weight amax equal what the streaming cast
// (cast_tma.cu) makes of the updated master: same conversions, same rules for
// values above the E4M3 range and for NaN payloads, the amax taken as the cast
// of the largest |p| (the fp32 value itself at the TF32 rung).
namespace apa {
namespace {

constexpr int kAR = 32;                         // tile rows
constexpr int kAC = 64;                         // tile columns: two 32-column boxes
constexpr int kAConsumerWarps = 16;           // one 16-byte chunk of the tile row per thread
constexpr int kAConsumers = 32 * kAConsumerWarps;
constexpr int kAThreads = kAConsumers + 32;
constexpr int kATensorBytes = kAR * kAC * 4;    // 8 KB of one fp32 tensor
constexpr int kAStageBytes = 4 * kATensorBytes; // p, g, m, v
constexpr int kAStages = 6;

template <int DST> struct AwCfg {
  static constexpr int ED = DST == APA_DT_E4M3 ? 1 : DST == APA_DT_F16 ? 2 : 4;
  static constexpr int kOutBytes = kAR * kAC * ED;   // one staging tile
  static constexpr int kSmemBytes = kAStages * kAStageBytes + 2 * kOutBytes + 2 * kAStages * 8 + 1024;
};

struct AdamwArgs {
  int64_t rows, cols;
  float* amax;
  int has_dst, has_dst_t, tf32;
  float decay, one_m_b1, b2, one_m_b2, eps, step_size, bc2_sqrt;
};

__device__ __forceinline__ void aw_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kAConsumers) : "memory"); }
__device__ __forceinline__ bool aw_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, 1, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(kAConsumers)
      : "memory");
  return r != 0;
}

// One element, in the order of torch.optim.AdamW's single-tensor update:
// p *= 1 - lr*wd; m += (1-b1)(g-m); v = v*b2 + g*g*(1-b2);
// p += -step_size * m / (sqrt(v)/sqrt(bc2) + eps).
__device__ __forceinline__ float aw_elem(float pv, float g, float& m, float& v, const AdamwArgs& a) {
  pv = __fmul_rn(pv, a.decay);
  m = __fadd_rn(m, __fmul_rn(a.one_m_b1, __fsub_rn(g, m)));
  v = __fadd_rn(__fmul_rn(v, a.b2), __fmul_rn(__fmul_rn(g, g), a.one_m_b2));
  const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), a.bc2_sqrt), a.eps);
  return __fadd_rn(pv, __fmul_rn(-a.step_size, __fdiv_rn(m, denom)));
}

template <int DST>
__global__ void __launch_bounds__(kAThreads, 1)
    adamw_cast_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmG,
                      const __grid_constant__ CUtensorMap tmM, const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmT, AdamwArgs a) {
  using C = AwCfg<DST>;
  constexpr int S = kAStages;
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = su32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* sStage = smem;                                 // S x {p, g, m, v}
  uint8_t* sOut = sStage + S * kAStageBytes;              // row-major staging
  uint8_t* sOutT = sOut + C::kOutBytes;                   // transposed staging
  uint64_t* full = reinterpret_cast<uint64_t*>(sOutT + C::kOutBytes);
  uint64_t* empty = full + S;
  __shared__ uint32_t red[kAThreads / 32];

  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int64_t tiles_r = (a.rows + kAR - 1) / kAR;
  const int64_t tiles_c = (a.cols + kAC - 1) / kAC;
  const int64_t ntiles = tiles_r * tiles_c;

  if (t == 0) {
    for (int s = 0; s < S; ++s) {
      cb_init(&full[s], 1);
      cb_init(&empty[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();   // the gradient and the optimizer state are final

  uint32_t mloc = 0;
  if (warp == kAConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int64_t tr = tile / tiles_c, tc = tile - tr * tiles_c;
        if (!cb_wait(&empty[stage], phase ^ 1u, kStatusTimeoutEmpty)) { ok = false; break; }
        cb_expect_tx(&full[stage], kAStageBytes);
        uint8_t* st = sStage + stage * kAStageBytes;
        const int x = (int)(tc * kAC), y = (int)(tr * kAR);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          ct_load(st + 0 * kATensorBytes + b * 4096, &tmP, x + 32 * b, y, &full[stage]);
          ct_load(st + 1 * kATensorBytes + b * 4096, &tmG, x + 32 * b, y, &full[stage]);
          ct_load(st + 2 * kATensorBytes + b * 4096, &tmM, x + 32 * b, y, &full[stage]);
          ct_load(st + 3 * kATensorBytes + b * 4096, &tmV, x + 32 * b, y, &full[stage]);
        }
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
    const int r = lane;                       // tile row
    const int box = warp >> 3;                // 32-column box
    const int kc = warp & 7;                  // 16-byte chunk in the box row
    const int c0 = 4 * warp;                  // first tile column
    int stage = 0, prev = -1;
    uint32_t phase = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int64_t tr = tile / tiles_c, tc = tile - tr * tiles_c;
      // a timed-out wait still runs the arithmetic on whatever the stage
      // holds; barrier B then ends the loop in every consumer
      const bool waited = cb_wait(&full[stage], phase, kStatusTimeoutFull);
      uint8_t* st = sStage + stage * kAStageBytes + box * 4096 + r * 128 + ((kc ^ (r & 7)) << 4);
      float4* pp = reinterpret_cast<float4*>(st + 0 * kATensorBytes);
      const float4 g4 = *reinterpret_cast<const float4*>(st + 1 * kATensorBytes);
      float4* mp = reinterpret_cast<float4*>(st + 2 * kATensorBytes);
      float4* vp = reinterpret_cast<float4*>(st + 3 * kATensorBytes);
      float4 p4 = *pp, m4 = *mp, v4 = *vp;
      p4.x = aw_elem(p4.x, g4.x, m4.x, v4.x, a);
      p4.y = aw_elem(p4.y, g4.y, m4.y, v4.y, a);
      p4.z = aw_elem(p4.z, g4.z, m4.z, v4.z, a);
      p4.w = aw_elem(p4.w, g4.w, m4.w, v4.w, a);
      *pp = p4;
      *mp = m4;
      *vp = v4;
      const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
      // amax over the elements inside the weight (the zero-filled margin can
      // hold NaN when eps is 0)
      const int64_t row = tr * kAR + r, col0 = tc * kAC + c0;
      uint32_t m = 0, tmax = 0;     // tmax: every element, for the choice of conversion path
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmax = max(tmax, mag_bits(pv[c]));
        if (row < a.rows && col0 + c < a.cols) m = max(m, mag_bits(pv[c]));
      }
      mloc = max(mloc, m);

      constexpr int W = C::ED;         // code words of the thread's 4 elements
      uint32_t code[W];
      if constexpr (DST == APA_DT_E4M3) {
        const bool big = tmax > kE4M3NaNThresholdBits;
        const uint32_t lo = big ? e4m3x2_exact(pv[0], pv[1]) : e4m3x2_sat(pv[0], pv[1]);
        const uint32_t hi = big ? e4m3x2_exact(pv[2], pv[3]) : e4m3x2_sat(pv[2], pv[3]);
        code[0] = lo | (hi << 16);
      } else if constexpr (DST == APA_DT_F16) {
        if (tmax > 0x7F800000u) {       // a NaN: keep sign and payload per element
#pragma unroll
          for (int k = 0; k < 2; ++k)
            code[k] = (uint32_t)f16_from_f32(pv[2 * k]) | ((uint32_t)f16_from_f32(pv[2 * k + 1]) << 16);
        } else {
#pragma unroll
          for (int k = 0; k < 2; ++k) code[k] = f16x2_from_f32(pv[2 * k], pv[2 * k + 1]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) code[k] = a.tf32 ? tf32_rn_bits(__float_as_uint(pv[k])) : __float_as_uint(pv[k]);
      }

      // the staging tiles of the previous tile must have been read by its
      // stores, and so must the previous stage (its p, m, v)
      if (t == 0) ct_wait_read0();
      // barrier B: every thread's in-place update is done, staging is free
      if (aw_sync_or(!waited)) break;
      if (t == 0 && prev >= 0) cb_arrive(&empty[prev]);

      if (a.has_dst) {
        if constexpr (DST == APA_DT_E4M3) {
          // 64-byte rows, 64-byte swizzle: bytes 4(w%4).. of chunk w/4
          *reinterpret_cast<uint32_t*>(sOut + r * 64 + (((warp >> 2) ^ ((r >> 1) & 3)) << 4) + 4 * (warp & 3)) =
              code[0];
        } else if constexpr (DST == APA_DT_F16) {
          // 128-byte rows, 128-byte swizzle: bytes 8(w%2).. of chunk w/2
          *reinterpret_cast<uint2*>(sOut + r * 128 + (((warp >> 1) ^ (r & 7)) << 4) + 8 * (warp & 1)) =
              make_uint2(code[0], code[1]);
        } else {
          // two 32-column boxes like the source tile
          *reinterpret_cast<uint4*>(sOut + box * 4096 + r * 128 + ((kc ^ (r & 7)) << 4)) =
              make_uint4(code[0], code[1], code[2], code[3]);
        }
      }
      if (a.has_dst_t) {
        // transposed tile: 64 rows (tile columns) of 32 elements (tile rows),
        // dense; a warp's store fills one 32-element row
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint8_t* dstp = sOutT + (c0 + c) * (32 * C::ED) + r * C::ED;
          if constexpr (DST == APA_DT_E4M3) {
            *dstp = (uint8_t)(code[0] >> (8 * c));
          } else if constexpr (DST == APA_DT_F16) {
            *reinterpret_cast<uint16_t*>(dstp) = (uint16_t)(code[c >> 1] >> (16 * (c & 1)));
          } else {
            *reinterpret_cast<uint32_t*>(dstp) = code[c];
          }
        }
      }
      ct_fence_smem();
      aw_sync();                                            // barrier A: stage and staging complete
      if (t == 0) {
        const int x = (int)(tc * kAC), y = (int)(tr * kAR);
        const uint8_t* sb = sStage + stage * kAStageBytes;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          if (x + 32 * b < a.cols) {
            ct_store(&tmP, sb + 0 * kATensorBytes + b * 4096, x + 32 * b, y);
            ct_store(&tmM, sb + 2 * kATensorBytes + b * 4096, x + 32 * b, y);
            ct_store(&tmV, sb + 3 * kATensorBytes + b * 4096, x + 32 * b, y);
          }
        }
        if (a.has_dst) {
          if constexpr (DST == APA_DT_F32) {
            ct_store(&tmD, sOut, x, y);
            if (x + 32 < a.cols) ct_store(&tmD, sOut + 4096, x + 32, y);
          } else {
            ct_store(&tmD, sOut, x, y);
          }
        }
        if (a.has_dst_t) ct_store(&tmT, sOutT, y, x);
        ct_commit();
      }
      prev = stage;
      if (++stage == S) { stage = 0; phase ^= 1u; }
    }
    // the last stage goes back once its stores have read it
    if (t == 0) {
      ct_wait_all0();
      if (prev >= 0) cb_arrive(&empty[prev]);
    }
  }

  // the working copy's amax is the cast of the largest |p|
  uint32_t mag = mloc;
  if constexpr (DST == APA_DT_E4M3) mag = e4m3_mag_bits(e4m3_from_f32(__uint_as_float(mloc)));
  else if constexpr (DST == APA_DT_F16) mag = mag_bits(f16_to_f32(f16_from_f32(__uint_as_float(mloc))));
  mag = warp_max_u32(mag);
  if (lane == 0) red[warp] = mag;
  __syncthreads();
  if (t < 32) {
    uint32_t mm = t < kAThreads / 32 ? red[t] : 0u;
    mm = warp_max_u32(mm);
    if (t == 0) telem_commit(a.amax, nullptr, mm);
  }
}

template <int DST>
int launch_adamw_cast_t(float* p, const float* g, float* m, float* v, int64_t rows, int64_t cols, int64_t ld,
                        void* wq, int64_t ld_q, void* wq_t, int64_t ld_qt, const AdamwArgs& args, cudaStream_t s) {
  using C = AwCfg<DST>;
  static std::once_flag once;
  static int blocks_per_sm = 0;
  std::call_once(once, [] {
    if (cudaFuncSetAttribute(adamw_cast_kernel<DST>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) !=
        cudaSuccess)
      return;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, adamw_cast_kernel<DST>, kAThreads, C::kSmemBytes) ==
        cudaSuccess)
      blocks_per_sm = n;
  });
  if (blocks_per_sm < 1) {
    (void)cudaGetLastError();
    return APA_ERR_UNSUPPORTED;
  }
  const CUtensorMapDataType ddt = DST == APA_DT_E4M3  ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                  : DST == APA_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapDataType f32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap mp, mg, mm, mv, md, mt;
  if (!cast_map(&mp, f32, p, cols, rows, ld * 4, 32, kAR, sw) || !cast_map(&mg, f32, g, cols, rows, ld * 4, 32, kAR, sw) ||
      !cast_map(&mm, f32, m, cols, rows, ld * 4, 32, kAR, sw) || !cast_map(&mv, f32, v, cols, rows, ld * 4, 32, kAR, sw))
    return APA_ERR_UNSUPPORTED;
  md = mp;
  mt = mp;
  if (wq) {
    const int bx = DST == APA_DT_F32 ? 32 : 64;
    const CUtensorMapSwizzle dsw = DST == APA_DT_E4M3 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    if (!cast_map(&md, ddt, wq, cols, rows, ld_q * C::ED, bx, kAR, dsw)) return APA_ERR_UNSUPPORTED;
  }
  if (wq_t) {
    if (!cast_map(&mt, ddt, wq_t, rows, cols, ld_qt * C::ED, kAR, kAC, CU_TENSOR_MAP_SWIZZLE_NONE))
      return APA_ERR_UNSUPPORTED;
  }
  AdamwArgs a = args;
  a.rows = rows;
  a.cols = cols;
  a.has_dst = wq != nullptr;
  a.has_dst_t = wq_t != nullptr;
  const int64_t tiles = ((rows + kAR - 1) / kAR) * ((cols + kAC - 1) / kAC);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)num_sms() * blocks_per_sm));
  if (launch_kernel(adamw_cast_kernel<DST>, dim3((unsigned)grid), dim3(kAThreads), C::kSmemBytes, s, 1, mp, mg, mm, mv,
                    md, mt, a) != cudaSuccess)
    return APA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

}  // namespace
}  // namespace apa

// AdamW on an fp32 master weight fused with the next step's working copy:
// p, m, v updated in place (torch.optim.AdamW order of operations, step >= 1)
// and, in the same pass, p cast to the working dtype into wq (row-major)
// and/or wq_t (transposed) with max |cast value| written to *w_amax. 16-byte
// aligned rows everywhere; APA_ERR_UNSUPPORTED otherwise (the caller then runs
// AdamW and the cast separately).
extern "C" int apa_adamw_cast(float* p, const float* g, float* m, float* v, int64_t rows, int64_t cols, int64_t ld,
                              float lr, float beta1, float beta2, float eps, float weight_decay, int64_t step,
                              void* wq, int work_dtype, int64_t ld_q, void* wq_t, int64_t ld_qt, float* w_amax,
                              void* stream) {
  using namespace apa;
  if (!p || !g || !m || !v || rows <= 0 || cols <= 0 || ld < cols || step < 1) return APA_ERR_INVALID;
  if (!wq && !wq_t) return APA_ERR_INVALID;
  const int tf32 = work_dtype == APA_DT_TF32;
  const int dst = tf32 ? APA_DT_F32 : work_dtype;
  if (dst != APA_DT_E4M3 && dst != APA_DT_F16 && dst != APA_DT_F32) return APA_ERR_UNSUPPORTED;
  const int ed = dst == APA_DT_E4M3 ? 1 : dst == APA_DT_F16 ? 2 : 4;
  if (!tma_ok(p, ld, 4) || !tma_ok(g, ld, 4) || !tma_ok(m, ld, 4) || !tma_ok(v, ld, 4)) return APA_ERR_UNSUPPORTED;
  if ((wq && !tma_ok(wq, ld_q, ed)) || (wq_t && !tma_ok(wq_t, ld_qt, ed))) return APA_ERR_UNSUPPORTED;
  if (rows >= (1ll << 31) || cols >= (1ll << 31)) return APA_ERR_UNSUPPORTED;
  AdamwArgs a;
  a.amax = w_amax;
  a.tf32 = tf32;
  const double bc1 = 1.0 - std::pow((double)beta1, (double)step);
  const double bc2 = 1.0 - std::pow((double)beta2, (double)step);
  a.decay = (float)(1.0 - (double)lr * (double)weight_decay);
  a.one_m_b1 = (float)(1.0 - (double)beta1);
  a.b2 = beta2;
  a.one_m_b2 = (float)(1.0 - (double)beta2);
  a.eps = eps;
  a.step_size = (float)((double)lr / bc1);
  a.bc2_sqrt = (float)std::sqrt(bc2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the working copy's amax starts over with each update
  if (w_amax && cudaMemsetAsync(w_amax, 0, sizeof(float), s) != cudaSuccess) return APA_ERR_CUDA;
  switch (dst) {
    case APA_DT_E4M3: return launch_adamw_cast_t<APA_DT_E4M3>(p, g, m, v, rows, cols, ld, wq, ld_q, wq_t, ld_qt, a, s);
    case APA_DT_F16: return launch_adamw_cast_t<APA_DT_F16>(p, g, m, v, rows, cols, ld, wq, ld_q, wq_t, ld_qt, a, s);
    default: return launch_adamw_cast_t<APA_DT_F32>(p, g, m, v, rows, cols, ld, wq, ld_q, wq_t, ld_qt, a, s);
  }
}
