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
//                        (skip); bit2: at least one module escalated
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

__global__ void ladder_eval_kernel(LadderArgs a) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int L = a.L, O = a.O;
  int* hdr = reinterpret_cast<int*>(a.out);
  int* code = hdr + 4;
  int* ocode = code + L;
  int* lvl_out = ocode + O;
  const int nint = 4 + 2 * L + O;
  double* dbl = reinterpret_cast<double*>(a.out + ((nint * 4 + 7) & ~7));
  double* ema_out = dbl;
  double* trig = dbl + L;
  double* otrig = trig + L;

  auto flag_of = [&](int i) -> bool { return a.global ? a.global[1 + i] > 0 : *a.flag[i] > 0; };
  auto amax_of = [&](int i) -> float { return a.global ? __int_as_float(a.global[1 + L + i]) : *a.amax[i]; };
  auto ratio_of = [&](int i) -> float { return a.global ? __int_as_float(a.global[1 + 2 * L + i]) : *a.ratio[i]; };
  auto oflag_of = [&](int j) -> bool { return a.global ? a.global[1 + 3 * L + j] > 0 : *a.oflag[j] > 0; };
  auto oamax_of = [&](int j) -> float { return a.global ? __int_as_float(a.global[1 + 3 * L + O + j]) : *a.oamax[j]; };

  bool hard = false;
  if (a.global) {
    hard = a.global[0] > 0;
  } else {
    for (int i = 0; i < L && !hard; ++i) hard = flag_of(i);
    for (int j = 0; j < O && !hard; ++j) hard = oflag_of(j);
  }
  const bool eval = hard || (a.interval > 0 && (a.step % a.interval) == 0);
  int status = 0;
  int min_level = 1;
  for (int i = 0; i < L; ++i) { code[i] = 0; trig[i] = 0.0; }
  for (int j = 0; j < O; ++j) { ocode[j] = 0; otrig[j] = 0.0; }
  if (eval) {
    status |= 1;
    bool overflow = false;
    for (int i = 0; i < L; ++i) {
      const double av = (double)amax_of(i);
      const bool nonf = flag_of(i);
      const int old = a.level[i];
      const double thr = thr_of(a, old);
      int reason = 0;
      double t = 0.0;
      if (nonf || isinf(av) || isnan(av) || av > thr) {
        overflow = true;
        reason = 1;
        t = (nonf && !isinf(av) && !isnan(av) && av <= thr) ? (double)NAN : av;
      } else {
        const double r = (double)ratio_of(i);
        // alpha * ema + (1 - alpha) * r, each operation rounded as Python does
        const double e = __dadd_rn(__dmul_rn(a.alpha, a.ema[i]), __dmul_rn(__dsub_rn(1.0, a.alpha), r));
        a.ema[i] = e;
        if (e > a.theta) {
          reason = 2;
          t = e;
        }
      }
      int c = 0;
      if (reason) {
        c = reason | (old << 4);
        if (old < 2) {
          a.level[i] = old + 1;
          a.ema[i] = 0.0;
          c |= 4;
          status |= 4;
        }
      }
      code[i] = c;
      trig[i] = t;
      // reset the window (manager.py:237-239); the pointers are the module's own buffers
      *a.amax[i] = 0.0f;
      *a.ratio[i] = 0.0f;
      *a.flag[i] = 0;
    }
    if (L > 0) {
      min_level = a.level[0];
      for (int i = 1; i < L; ++i) min_level = min(min_level, a.level[i]);
    }
    const double othr = thr_of(a, min_level);
    for (int j = 0; j < O; ++j) {
      const double av = (double)oamax_of(j);
      const bool nonf = oflag_of(j);
      if (nonf || isinf(av) || isnan(av) || av > othr) {
        overflow = true;
        ocode[j] = 1;
        otrig[j] = (nonf && !isinf(av) && !isnan(av)) ? (double)NAN : av;
      }
      *a.oamax[j] = 0.0f;
      *a.oflag[j] = 0;
    }
    if (overflow) status |= 2;
  }
  for (int i = 0; i < L; ++i) {
    lvl_out[i] = a.level[i];
    ema_out[i] = a.ema[i];
  }
  hdr[0] = status;
  hdr[1] = min_level;
  hdr[2] = L;
  hdr[3] = O;
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
  ladder_pack_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      L, amax_ptr, ratio_ptr, reinterpret_cast<const int* const*>(flag_ptr), O, oamax_ptr,
      reinterpret_cast<const int* const*>(oflag_ptr), reinterpret_cast<int*>(packed));
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

extern "C" int apa_ladder_eval(int L, float* const* amax_ptr, float* const* ratio_ptr, int32_t* const* flag_ptr,
                               int32_t* level, double* ema, int O, float* const* oamax_ptr,
                               int32_t* const* oflag_ptr, const int32_t* global, int64_t step_count,
                               int64_t check_interval, double theta, double alpha, void* out, void* stream) {
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
  ladder_eval_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}
