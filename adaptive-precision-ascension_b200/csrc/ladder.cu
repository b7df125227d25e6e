// K5: the escalation ladder evaluated on the device.
//
// Reproduces APAManager._check_hard_overflow (manager.py:178-189),
// _do_full_evaluation (manager.py:206-261) and the level/EMA half of
// _escalate_module (manager.py:267-293) for all modules in one launch. The
// per-module decisions depend on each other only through the minimum APA
// level used for the non-APA checks, and the reference walks modules in
// registration order, so a single thread walks them in that order too: the
// work is O(modules) scalar compares, far below a microsecond.
//
// Decision record written to `out` (read by the host in one copy):
//   int32  hdr[4]        {status bits, min_level, L, O}
//                        status bit0: evaluation ran; bit1: batch has overflow
//                        (skip); bit2: at least one module escalated; bit8:
//                        the library status word is set (a bounded wait of
//                        some earlier kernel gave up)
//   int32  code[L]       bits 0-1 reason (1 OVERFLOW, 2 SILENT_UNDERFLOW),
//                        bit 2 escalated, bits 4-5 level before
//   int32  ocode[O]      1 when the non-APA leaf overflowed
//   int32  level[L]      level after this step
//   (padding to 8 bytes)
//   double ema[L]        EMA after this step
//   double trig[L]       trigger value (reference semantics, may be NaN)
//   double otrig[O]
#include "apa_common.cuh"

namespace apa {
namespace {

struct LadderArgs {
  int L, O;
  float* const* amax; float* const* ratio; int* const* flag;
  int* level; double* ema;
  float* const* oamax; int* const* oflag;
  const int* global;
  long long step, interval;
  double theta, alpha;
  double thr0, thr1, thr2;
  char* out;
};

__device__ __forceinline__ double thr_of(const LadderArgs& a, int lvl) {
  return lvl == 0 ? a.thr0 : lvl == 1 ? a.thr1 : lvl == 2 ? a.thr2 : (double)INFINITY;
}

__global__ void ladder_pack_kernel(int L, const float* const* amax, const float* const* ratio, const int* const* flag,
                                   int O, const float* const* oamax, const int* const* oflag, int* packed) {
  pdl_launch_dependents();
  pdl_wait();
  // [hard][flag L][amax bits L][ratio bits L][oflag O][oamax bits O]; all
  // entries reduce correctly under an int32 MAX across ranks (non-negative
  // floats and NaN order like their bit patterns).
  const int tid = threadIdx.x;
  __shared__ int any;
  if (tid == 0) any = 0;
  __syncthreads();
  for (int i = tid; i < L; i += blockDim.x) {
    const int f = *flag[i] > 0 ? 1 : 0;
    packed[1 + i] = f;
    packed[1 + L + i] = __float_as_int(*amax[i]);
    packed[1 + 2 * L + i] = __float_as_int(*ratio[i]);
    if (f) atomicOr(&any, 1);
  }
  for (int j = tid; j < O; j += blockDim.x) {
    const int f = *oflag[j] > 0 ? 1 : 0;
    packed[1 + 3 * L + j] = f;
    packed[1 + 3 * L + O + j] = __float_as_int(*oamax[j]);
    if (f) atomicOr(&any, 1);
  }
  __syncthreads();
  if (tid == 0) packed[0] = any;
}

// Shared-memory image of the per-module state, filled by all threads so the
// dependent global loads overlap; one thread then walks the modules in order.
__global__ void __launch_bounds__(256) ladder_eval_kernel(LadderArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ double sh_d[];
  const int L = a.L, O = a.O;
  double* s_ema = sh_d;                                        // [L]
  double* s_trig = s_ema + L;                                  // [L]
  double* s_otrig = s_trig + L;                                // [O]
  float* s_amax = reinterpret_cast<float*>(s_otrig + O);       // [L]
  float* s_ratio = s_amax + L;                                 // [L]
  float* s_oamax = s_ratio + L;                                // [O]
  int* s_flag = reinterpret_cast<int*>(s_oamax + O);           // [L]
  int* s_level = s_flag + L;                                   // [L]
  int* s_code = s_level + L;                                   // [L]
  int* s_oflag = s_code + L;                                   // [O]
  int* s_ocode = s_oflag + O;                                  // [O]
  __shared__ int s_hdr[2];
  const int tid = threadIdx.x;

  for (int i = tid; i < L; i += blockDim.x) {
    if (a.global) {
      s_flag[i] = a.global[1 + i] > 0;
      s_amax[i] = __int_as_float(a.global[1 + L + i]);
      s_ratio[i] = __int_as_float(a.global[1 + 2 * L + i]);
    } else {
      s_flag[i] = *a.flag[i] > 0;
      s_amax[i] = *a.amax[i];
      s_ratio[i] = *a.ratio[i];
    }
    s_level[i] = a.level[i];
    s_ema[i] = a.ema[i];
    s_code[i] = 0;
    s_trig[i] = 0.0;
  }
  for (int j = tid; j < O; j += blockDim.x) {
    if (a.global) {
      s_oflag[j] = a.global[1 + 3 * L + j] > 0;
      s_oamax[j] = __int_as_float(a.global[1 + 3 * L + O + j]);
    } else {
      s_oflag[j] = *a.oflag[j] > 0;
      s_oamax[j] = *a.oamax[j];
    }
    s_ocode[j] = 0;
    s_otrig[j] = 0.0;
  }
  __syncthreads();

  if (tid == 0) {
    bool hard = false;
    if (a.global) {
      hard = a.global[0] > 0;
    } else {
      for (int i = 0; i < L && !hard; ++i) hard = s_flag[i];
      for (int j = 0; j < O && !hard; ++j) hard = s_oflag[j];
    }
    const bool eval = hard || (a.interval > 0 && (a.step % a.interval) == 0);
    int status = 0;
    int min_level = 1;
    if (eval) {
      status |= 1;
      bool overflow = false;
      for (int i = 0; i < L; ++i) {
        const double av = (double)s_amax[i];
        const bool nonf = s_flag[i] != 0;
        const int old = s_level[i];
        const double thr = thr_of(a, old);
        int reason = 0;
        double t = 0.0;
        if (nonf || isinf(av) || isnan(av) || av > thr) {
          overflow = true;
          reason = 1;
          t = (nonf && !isinf(av) && !isnan(av) && av <= thr) ? (double)NAN : av;
        } else {
          const double r = (double)s_ratio[i];
          // alpha * ema + (1 - alpha) * r, each operation rounded as Python does
          const double e = __dadd_rn(__dmul_rn(a.alpha, s_ema[i]), __dmul_rn(__dsub_rn(1.0, a.alpha), r));
          s_ema[i] = e;
          if (e > a.theta) {
            reason = 2;
            t = e;
          }
        }
        int c = 0;
        if (reason) {
          c = reason | (old << 4);
          if (old < 2) {
            s_level[i] = old + 1;
            s_ema[i] = 0.0;
            c |= 4;
            status |= 4;
          }
        }
        s_code[i] = c;
        s_trig[i] = t;
      }
      if (L > 0) {
        min_level = s_level[0];
        for (int i = 1; i < L; ++i) min_level = min(min_level, s_level[i]);
      }
      const double othr = thr_of(a, min_level);
      for (int j = 0; j < O; ++j) {
        const double av = (double)s_oamax[j];
        const bool nonf = s_oflag[j] != 0;
        if (nonf || isinf(av) || isnan(av) || av > othr) {
          overflow = true;
          s_ocode[j] = 1;
          s_otrig[j] = (nonf && !isinf(av) && !isnan(av)) ? (double)NAN : av;
        }
      }
      if (overflow) status |= 2;
    }
    s_hdr[0] = status;
    s_hdr[1] = min_level;
  }
  __syncthreads();

  const int status = s_hdr[0];
  int* hdr = reinterpret_cast<int*>(a.out);
  int* code = hdr + 4;
  int* ocode = code + L;
  int* lvl_out = ocode + O;
  const int nint = 4 + 2 * L + O;
  double* dbl = reinterpret_cast<double*>(a.out + ((nint * 4 + 7) & ~7));
  double* ema_out = dbl;
  double* trig = dbl + L;
  double* otrig = trig + L;
  for (int i = tid; i < L; i += blockDim.x) {
    a.level[i] = s_level[i];
    a.ema[i] = s_ema[i];
    lvl_out[i] = s_level[i];
    ema_out[i] = s_ema[i];
    code[i] = s_code[i];
    trig[i] = s_trig[i];
    if (status & 1) {
      // reset the window (manager.py:237-239); the pointers are the module's own buffers
      *a.amax[i] = 0.0f;
      *a.ratio[i] = 0.0f;
      *a.flag[i] = 0;
    }
  }
  for (int j = tid; j < O; j += blockDim.x) {
    ocode[j] = s_ocode[j];
    otrig[j] = s_otrig[j];
    if (status & 1) {
      *a.oamax[j] = 0.0f;
      *a.oflag[j] = 0;
    }
  }
  if (tid == 0) {
    hdr[0] = status | (g_status != 0u ? 0x100 : 0);
    hdr[1] = s_hdr[1];
    hdr[2] = L;
    hdr[3] = O;
  }
}

size_t ladder_smem_bytes(int L, int O) {
  return (size_t)(2 * L + O) * sizeof(double) + (size_t)(2 * L + O) * sizeof(float) + (size_t)(3 * L + 2 * O) * sizeof(int);
}

size_t ladder_record_bytes(int L, int O) {
  const size_t nint = 4 + 2 * (size_t)L + O;
  return ((nint * 4 + 7) & ~(size_t)7) + 8 * (2 * (size_t)L + O);
}

}  // namespace
}  // namespace apa

using namespace apa;

extern "C" int apa_abi_version(void) { return 1; }

extern "C" const char* apa_status_string(int status) {
  switch (status) {
    case APA_OK: return "ok";
    case APA_ERR_INVALID: return "invalid argument (null pointer, bad size or leading dimension)";
    case APA_ERR_ALIGN: return "operand not 16-byte aligned for the TMA path";
    case APA_ERR_UNSUPPORTED: return "unsupported dtype or rung";
    case APA_ERR_CUDA: return "CUDA launch or driver error";
    case APA_ERR_NOALLOC_LIMIT:
      return "problem exceeds the no-allocation scratch (ceil(rows/64) * cols must be <= 4194304)";
    default: return "unknown status";
  }
}

extern "C" int apa_ladder_pack(int L, const float* const* amax_ptr, const float* const* ratio_ptr,
                               const int32_t* const* flag_ptr, int O, const float* const* oamax_ptr,
                               const int32_t* const* oflag_ptr, int32_t* packed, void* stream) {
  if (L < 0 || O < 0 || !packed) return APA_ERR_INVALID;
  if ((L > 0 && (!amax_ptr || !ratio_ptr || !flag_ptr)) || (O > 0 && (!oamax_ptr || !oflag_ptr)))
    return APA_ERR_INVALID;
  apa::launch_kernel(apa::ladder_pack_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), 1, L, amax_ptr,
                     ratio_ptr, reinterpret_cast<const int* const*>(flag_ptr), O, oamax_ptr,
                     reinterpret_cast<const int* const*>(oflag_ptr), reinterpret_cast<int*>(packed));
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_ladder_eval(int L, float* const* amax_ptr, float* const* ratio_ptr, int32_t* const* flag_ptr,
                               int32_t* level, double* ema, int O, float* const* oamax_ptr,
                               int32_t* const* oflag_ptr, const int32_t* global, int64_t step_count,
                               int64_t check_interval, double theta, double alpha, void* out, void* out_host,
                               void* stream) {
  if (L < 0 || O < 0 || !out) return APA_ERR_INVALID;
  if ((L > 0 && (!amax_ptr || !ratio_ptr || !flag_ptr || !level || !ema)) || (O > 0 && (!oamax_ptr || !oflag_ptr)))
    return APA_ERR_INVALID;
  LadderArgs a;
  a.L = L; a.O = O;
  a.amax = amax_ptr; a.ratio = ratio_ptr; a.flag = reinterpret_cast<int* const*>(flag_ptr);
  a.level = reinterpret_cast<int*>(level); a.ema = ema;
  a.oamax = oamax_ptr; a.oflag = reinterpret_cast<int* const*>(oflag_ptr);
  a.global = reinterpret_cast<const int*>(global);
  a.step = step_count; a.interval = check_interval;
  a.theta = theta; a.alpha = alpha;
  // THRESHOLDS_MAX (config.py:9-13) evaluated exactly as Python does
  a.thr0 = 0.90 * 448.0;
  a.thr1 = 0.90 * 65504.0;
  a.thr2 = (double)INFINITY;
  a.out = static_cast<char*>(out);
  const size_t smem = ladder_smem_bytes(L, O);
  if (smem > 200 * 1024) return APA_ERR_INVALID;   // far beyond any model's module count
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(ladder_eval_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return APA_ERR_CUDA;
  }
  apa::launch_kernel(apa::ladder_eval_kernel, dim3(1), dim3(256), smem, st, 1, a);
  if (cudaGetLastError() != cudaSuccess) return APA_ERR_CUDA;
  if (out_host != nullptr &&
      cudaMemcpyAsync(out_host, out, ladder_record_bytes(L, O), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return APA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}
