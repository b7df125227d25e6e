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
//   warps 2..9  epilogue: two warps per TMEM lane quarter, each taking half
//               of the tile's columns; tcgen05.ld 32 lanes x 32 columns at a
//               time, apply the op's epilogue, stage 32 x 128-byte boxes in a
//               small ring of shared-memory buffers and write them with TMA
//               bulk-tensor stores; the accumulator is double buffered so the
//               epilogue of tile i overlaps the MMAs of i+1.
//
// CTA-pair variant (PAIR): a cluster of two CTAs on two SMs computes a
// 256 x BN tile with tcgen05.mma.cta_group::2 (M = 256). Each CTA loads its
// own 128 rows of A and half (BN/2 rows) of B, so per output element the
// pair reads 1.5x fewer operand bytes from L2 than two single CTAs. Both
// CTAs' loads complete on the even CTA's full barrier (the even CTA expects
// the bytes of both); the even CTA's one MMA thread issues the MMAs, which
// read both CTAs' shared memory and write each CTA's 128 accumulator rows into
// its own TMEM; tcgen05.commit multicasts the stage release and the
// accumulator-ready signal to both CTAs; both CTAs' epilogue warps hand the
// accumulator back on the even CTA's barrier. Operand loads are plain
// (non-multicast) TMA loads.
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
#include "dp_region.cuh"

namespace apa {
int num_sms();
namespace gemm {

constexpr int BM = 128;
constexpr int kSlab = 128;            // K bytes per pipeline stage (one swizzle row)
// Epilogue warps EW = 4 or 8: warp w may only read TMEM lanes 32*(w%4) ..
// +31, so each lane quarter (32 accumulator rows) gets EW/4 warps that split
// the tile's columns between them. 8 warps when the epilogue cannot hide
// behind the next tile's MMAs (short K, or one or two tiles per CTA); 4 warps
// and a deeper operand pipeline otherwise.
template <int EW> constexpr int threads_for() { return 64 + 32 * EW; }


enum { KIND_E4M3 = 0, KIND_F16 = 1, KIND_TF32 = 2 };
// EPI_RAW: the fp32 accumulator as is (split-K partial sums, bare timing)
enum { EPI_FWD = 0, EPI_DGRAD = 1, EPI_WGRAD = 2, EPI_RAW = 3 };

template <int KIND> struct KindInfo;
template <> struct KindInfo<KIND_E4M3> { static constexpr int bytes = 1; static constexpr uint32_t fmt = 0; };
template <> struct KindInfo<KIND_F16> { static constexpr int bytes = 2; static constexpr uint32_t fmt = 0; };
template <> struct KindInfo<KIND_TF32> { static constexpr int bytes = 4; static constexpr uint32_t fmt = 2; };

constexpr int kEpiStageBytes = 4096;   // one staging buffer: 32 rows x 128 bytes of output


// BN: N extent of the output tile; with PAIR each CTA loads BN/2 rows of B.
// Pipeline depth and staging buffers per epilogue warp, per shape: the
// staging ring lets a warp fill the next buffer while earlier TMA stores are
// still reading theirs.
template <int BN, bool PAIR, int EW> struct Cfg {
  static constexpr int kCtas = PAIR ? 2 : 1;
  static constexpr int kTileM = BM * kCtas;
  static constexpr int kBRows = BN / kCtas;
  static constexpr int kABytes = BM * kSlab;
  static constexpr int kBBytes = kBRows * kSlab;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = EW == 8 ? (PAIR ? 4 : (BN == 256 ? 3 : 4)) : (PAIR ? 6 : (BN == 256 ? 4 : 6));
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kEpiWarps = EW;
  static constexpr int kEpiThreads = 32 * EW;
  static constexpr int kThreads = threads_for<EW>();
  static constexpr int kEpiBufs = EW == 8 ? 2 : 1;
  static constexpr int kWarpCols = BN / (EW / 4);                      // columns per epilogue warp
  static constexpr int kEpiBytes = EW * kEpiBufs * kEpiStageBytes + EW * kWarpCols * 4;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + kBarrierBytes + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct EpiArgs {
  void* out; int64_t ldo; int out_dt; int vec_out;
  int tma_out;                      // output written by TMA bulk-tensor stores
  int coalesced_out;                // output written by store_box_coalesced
  const void* bias;                 // FWD: working-dtype bias (nullable)
  int bias_vec;                     // FWD: bias aligned for one vector load per 4 columns
  float* amax; int* flag;           // FWD: module telemetry; DGRAD: boundary_cast telemetry
  unsigned long long* counters;     // WGRAD: [nonzero, underflow, ticket], zero on entry
  float* ratio_max;                 // WGRAD: module gpu_underflow_ratio
  float vmin;                       // WGRAD: underflow threshold as fp32
  int accumulate;                   // WGRAD: add into out instead of overwriting
  int finalize;                     // WGRAD: form the ratio from the counts (0: leave them for a later block)
  int telem;                        // 0: no telemetry buffers, skip the telemetry-only work
  int splits;                       // split-K: K blocks divided into this many units per tile
  int kb_per_split;                 // 128-byte K slabs per split
  int split_rows;                   // output row offset between the splits' slices
  // stream-K tail: tiles from sk_first on (the last, partial wave) are split
  // along K into sk_splits = 2 units that run in the same wave; each
  // epilogue warp stores its raw partial to sk_ws and takes a ticket, and the
  // warp that finishes second adds the other partial and applies the
  // epilogue. sk_splits < 2: no tail split.
  float* sk_ws;                     // [tail tile][split][cta][epi warp][cols/4][32 lanes][4] fp32
  int* sk_tickets;                  // [tail tile][cta][epi warp], zero on entry and on exit
  int64_t sk_ws_bytes;              // caller workspace available (partials + tickets)
  int sk_first, sk_splits, sk_kb_per_split;
  // WGRAD: the data-parallel average of the output run in the epilogue
  // (dp.mc null: off): every warp publishes its 32 x 64 regions once they
  // are stored and averages the ones this rank owns across the ranks
  dpr::RegionArgs dp;
  int M, N, K;
};

// One work unit of the persistent schedule: an output tile and the range of
// 128-byte K slabs it reduces. sk_split >= 0 marks a stream-K tail unit;
// orow is the output row offset of a split-K slice.
struct Unit {
  int tile, kb0, kb1, sk_split, orow;
};

__host__ __device__ __forceinline__ int num_work_units(const EpiArgs& ea, int num_tiles) {
  if (ea.sk_splits > 1) return ea.sk_first + (num_tiles - ea.sk_first) * ea.sk_splits;
  return num_tiles * (ea.splits > 1 ? ea.splits : 1);
}

__device__ __forceinline__ Unit unit_of(const EpiArgs& ea, int w, int kb_count) {
  Unit u;
  u.sk_split = -1;
  u.orow = 0;
  if (ea.sk_splits > 1 && w >= ea.sk_first) {
    const int v = w - ea.sk_first;
    u.tile = ea.sk_first + v / ea.sk_splits;
    u.sk_split = v - (v / ea.sk_splits) * ea.sk_splits;
    u.kb0 = u.sk_split * ea.sk_kb_per_split;
    u.kb1 = min(u.kb0 + ea.sk_kb_per_split, kb_count);
  } else if (ea.splits > 1) {
    u.tile = w / ea.splits;
    const int sp = w - u.tile * ea.splits;
    u.kb0 = sp * ea.kb_per_split;
    u.kb1 = min(u.kb0 + ea.kb_per_split, kb_count);
    u.orow = sp * ea.split_rows;
  } else {
    u.tile = w;
    u.kb0 = 0;
    u.kb1 = kb_count;
  }
  return u;
}

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

// CLUSTER: acquire at cluster scope, for barriers the peer CTA arrives on.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (CLUSTER) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  }
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false after ~2 s.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int why) {
  if (mbar_try_wait<CLUSTER>(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait<CLUSTER>(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      atomicOr(&g_status, why);
      return false;
    }
  }
  return true;
}

// --- cluster (CTA pair) helpers ---
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster; orders shared-memory writes
// (barrier init, the TMEM address) before the peer's first access.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_cta(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// CTA-pair load: data into this CTA's shared memory, completion signalled on
// the mbarrier at `bar_cluster` (the even CTA's barrier). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* tm, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar_cluster)
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
template <int KIND, int BN, int TM = BM>
__host__ __device__ constexpr uint32_t idesc() {
  return (1u << 4) | (KindInfo<KIND>::fmt << 7) | (KindInfo<KIND>::fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(TM >> 4) << 24);
}

template <int KIND, bool PAIR = false>
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
  if constexpr (PAIR) {
    if constexpr (KIND == KIND_E4M3) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
          "l"(a), "l"(b), "r"(id), "r"(accumulate));
    } else if constexpr (KIND == KIND_F16) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
          "l"(a), "l"(b), "r"(id), "r"(accumulate));
    } else {
      asm volatile(
          "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
          "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
          "l"(a), "l"(b), "r"(id), "r"(accumulate));
    }
  } else if constexpr (KIND == KIND_E4M3) {
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

template <bool PAIR = false>
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  if constexpr (PAIR) {
    // arrive on the barrier at this offset in both CTAs of the pair
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)0x3)
        : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
  }
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
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t bf16x2_from_f32(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float fu(uint32_t u) { return __uint_as_float(u); }

struct EpiState {
  uint32_t mag = 0;          // max |value| as fp32 bits, before the output rounding
  uint32_t nz = 0, uf = 0;   // WGRAD counters
};

// Telemetry reductions are taken on the unrounded fp32 values: rounding to
// E4M3 / fp16 is monotone in magnitude (including the NaN rule above 464),
// so max |round(v)| = round(max |v|) and one conversion at the end suffices.
__device__ __forceinline__ uint32_t chunk_max(const uint32_t* r, int n, bool check, bool row_ok, int nv) {
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < 64; ++j) {
    if (j < n) {
      const uint32_t a = r[j] & 0x7FFFFFFFu;
      if (!check || (row_ok && j < nv)) m = max(m, a);
    }
  }
  return m;
}

// max(|a|, |b|, m), NaN-propagating: PTX max.NaN returns the canonical NaN
// (bits 0x7FFFFFFF) when an operand is NaN, which orders above every
// magnitude as the NaN's own bits do in the bit-pattern max of chunk_max;
// for all other values the result is the same float.
__device__ __forceinline__ float amax3(float a, float b, float m) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(fabsf(a)), "f"(fabsf(b)), "f"(m));
  return r;
}

// chunk_max of a whole 64-value chunk (no masking): two independent chains
// of three-input maxima.
__device__ __forceinline__ uint32_t chunk_max_full(const uint32_t* r) {
  float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
  for (int j = 0; j < 64; j += 4) {
    m0 = amax3(fu(r[j]), fu(r[j + 1]), m0);
    m1 = amax3(fu(r[j + 2]), fu(r[j + 3]), m1);
  }
  float m;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(m) : "f"(m0), "f"(m1));
  return __float_as_uint(m);
}

// x0 += b0, x1 += b1 (fp32 words) in one packed instruction; add.rn.f32x2
// rounds each lane exactly as add.rn.f32 does.
__device__ __forceinline__ void add2(uint32_t& x0, uint32_t& x1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\t"
      "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "+r"(x0), "+r"(x1)
      : "r"(__float_as_uint(b0)), "r"(__float_as_uint(b1)));
}

// The forward's bias for one epilogue warp's columns, in two halves: the raw
// working-dtype words of 4 columns per lane (one vector load when aligned),
// loaded one tile ahead so the load's latency hides behind the previous
// tile's epilogue, then converted to fp32 into the warp's bias row in shared
// memory. Columns past N read as +0.
template <int WARP_COLS>
struct BiasRaw {
  static constexpr int kRounds = (WARP_COLS + 127) / 128;
  uint32_t w[kRounds][4];
};

template <int KIND, int WARP_COLS>
__device__ __forceinline__ void bias_load(const EpiArgs& ea, int col_base, int lane, BiasRaw<WARP_COLS>& br) {
  constexpr int es = KindInfo<KIND>::bytes;
#pragma unroll
  for (int j = 0; j < BiasRaw<WARP_COLS>::kRounds; ++j) {
    const int c = 128 * j + 4 * lane;
    br.w[j][0] = br.w[j][1] = br.w[j][2] = br.w[j][3] = 0u;
    if (c >= WARP_COLS) continue;
    const int n = col_base + c;
    const uint8_t* p = static_cast<const uint8_t*>(ea.bias) + (int64_t)n * es;
    if (ea.bias_vec && n + 4 <= ea.N) {
      if constexpr (es == 1) {
        br.w[j][0] = *reinterpret_cast<const uint32_t*>(p);
      } else if constexpr (es == 2) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        br.w[j][0] = v.x; br.w[j][1] = v.y;
      } else {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        br.w[j][0] = v.x; br.w[j][1] = v.y; br.w[j][2] = v.z; br.w[j][3] = v.w;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (n + e >= ea.N) break;
        if constexpr (es == 1) br.w[j][0] |= (uint32_t)p[e] << (8 * e);
        else if constexpr (es == 2) br.w[j][e >> 1] |= (uint32_t)reinterpret_cast<const uint16_t*>(p)[e] << (16 * (e & 1));
        else br.w[j][e] = reinterpret_cast<const uint32_t*>(p)[e];
      }
    }
  }
}

template <int KIND, int WARP_COLS>
__device__ __forceinline__ void bias_store(float* sb, int lane, const BiasRaw<WARP_COLS>& br) {
#pragma unroll
  for (int j = 0; j < BiasRaw<WARP_COLS>::kRounds; ++j) {
    const int c = 128 * j + 4 * lane;
    if (c >= WARP_COLS) continue;
    float4 f;
    if constexpr (KIND == KIND_E4M3) {
      f = make_float4(e4m3_to_f32(br.w[j][0] & 0xFFu), e4m3_to_f32((br.w[j][0] >> 8) & 0xFFu),
                      e4m3_to_f32((br.w[j][0] >> 16) & 0xFFu), e4m3_to_f32(br.w[j][0] >> 24));
    } else if constexpr (KIND == KIND_F16) {
      f = make_float4(f16_to_f32((uint16_t)(br.w[j][0] & 0xFFFFu)), f16_to_f32((uint16_t)(br.w[j][0] >> 16)),
                      f16_to_f32((uint16_t)(br.w[j][1] & 0xFFFFu)), f16_to_f32((uint16_t)(br.w[j][1] >> 16)));
    } else {
      f = make_float4(fu(br.w[j][0]), fu(br.w[j][1]), fu(br.w[j][2]), fu(br.w[j][3]));
    }
    *reinterpret_cast<float4*>(sb + c) = f;
  }
}

// One 64-column unit of one row: r[0..63] hold the fp32 accumulators on
// entry and the output words on exit (64 fp32 words, or 32 words of packed
// 16-bit pairs). check: the tile is ragged, mask telemetry with row_ok / nv.
template <int KIND, int EPI>
__device__ __forceinline__ void epi_unit(const EpiArgs& ea, const float* sb, uint32_t (&r)[64], EpiState& st,
                                         bool check, bool row_ok, int nv) {
  if constexpr (EPI == EPI_FWD) {
    if (ea.bias != nullptr) {
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const float4 b = reinterpret_cast<const float4*>(sb)[q];
        add2(r[4 * q + 0], r[4 * q + 1], b.x, b.y);
        add2(r[4 * q + 2], r[4 * q + 3], b.z, b.w);
      }
    }
    if (ea.telem) st.mag = max(st.mag, check ? chunk_max(r, 64, check, row_ok, nv) : chunk_max_full(r));
    if constexpr (KIND == KIND_F16) {
#pragma unroll
      for (int k = 0; k < 32; ++k) r[k] = f16x2_from_f32(fu(r[2 * k]), fu(r[2 * k + 1]));
    }
  } else if constexpr (EPI == EPI_DGRAD) {
    // the chunk max also selects the E4M3 conversion (NaN rule above 464)
    const uint32_t m =
        (KIND == KIND_E4M3 || ea.telem) ? (check ? chunk_max(r, 64, check, row_ok, nv) : chunk_max_full(r)) : 0u;
    if (ea.telem) st.mag = max(st.mag, m);
    const int od = ea.out_dt;
    if constexpr (KIND == KIND_E4M3) {
      const bool big = __any_sync(0xFFFFFFFFu, m > kE4M3NaNThresholdBits);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float v0 = fu(r[2 * k]), v1 = fu(r[2 * k + 1]);
        const uint32_t h = f16x2_from_e4m3x2(big ? e4m3x2_exact(v0, v1) : e4m3x2_sat(v0, v1));
        if (od == APA_DT_F16) {
          r[k] = h;
        } else {
          const float f0 = f16lo_to_f32(h), f1 = f16hi_to_f32(h);
          if (od == APA_DT_BF16) {
            r[k] = (__float_as_uint(f0) >> 16) | (__float_as_uint(f1) & 0xFFFF0000u);   // exact
          } else {
            r[2 * k] = __float_as_uint(f0);
            r[2 * k + 1] = __float_as_uint(f1);
          }
        }
      }
    } else if constexpr (KIND == KIND_F16) {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const uint32_t h = f16x2_from_f32(fu(r[2 * k]), fu(r[2 * k + 1]));
        if (od == APA_DT_F16) {
          r[k] = h;
        } else if (od == APA_DT_BF16) {
          r[k] = bf16x2_from_f32(f16lo_to_f32(h), f16hi_to_f32(h));
        } else {
          r[2 * k] = __float_as_uint(f16lo_to_f32(h));
          r[2 * k + 1] = __float_as_uint(f16hi_to_f32(h));
        }
      }
    } else {
      if (od == APA_DT_BF16) {
#pragma unroll
        for (int k = 0; k < 32; ++k) r[k] = bf16x2_from_f32(fu(r[2 * k]), fu(r[2 * k + 1]));
      } else if (od == APA_DT_F16) {
#pragma unroll
        for (int k = 0; k < 32; ++k) r[k] = f16x2_from_f32(fu(r[2 * k]), fu(r[2 * k + 1]));
      }
    }
  } else if constexpr (EPI == EPI_RAW) {
    // raw fp32 accumulator: nothing to apply
  } else {
    const uint32_t vb = __float_as_uint(ea.vmin);
    if constexpr (KIND == KIND_E4M3) {
      const uint32_t m = check ? chunk_max(r, 64, check, row_ok, nv) : chunk_max_full(r);
      if (ea.telem) {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          // nonzero: 0 < |v| <= Inf (NaN excluded); underflow: nonzero and |v| < vmin
          const uint32_t a = (r[j] & 0x7FFFFFFFu) - 1u;
          const bool ok = !check || (row_ok && j < nv);
          st.nz += (ok && a < 0x7F800000u) ? 1u : 0u;
          st.uf += (ok && a < vb - 1u) ? 1u : 0u;
        }
      }
      const bool big = __any_sync(0xFFFFFFFFu, m > kE4M3NaNThresholdBits);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float v0 = fu(r[2 * k]), v1 = fu(r[2 * k + 1]);
        const uint32_t h = f16x2_from_e4m3x2(big ? e4m3x2_exact(v0, v1) : e4m3x2_sat(v0, v1));
        r[2 * k] = __float_as_uint(f16lo_to_f32(h));
        r[2 * k + 1] = __float_as_uint(f16hi_to_f32(h));
      }
    } else if constexpr (KIND == KIND_F16) {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const uint32_t h = f16x2_from_f32(fu(r[2 * k]), fu(r[2 * k + 1]));
        r[2 * k] = __float_as_uint(f16lo_to_f32(h));
        r[2 * k + 1] = __float_as_uint(f16hi_to_f32(h));
      }
      if (ea.telem) {
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const uint32_t a = (r[j] & 0x7FFFFFFFu) - 1u;
          const bool ok = !check || (row_ok && j < nv);
          st.nz += (ok && a < 0x7F800000u) ? 1u : 0u;
          st.uf += (ok && a < vb - 1u) ? 1u : 0u;
        }
      }
    }
  }
}

// Final telemetry magnitude: the unrounded max passed through the same
// rounding the stored (or hooked) tensor saw.
template <int KIND, int EPI>
__device__ __forceinline__ uint32_t final_mag(uint32_t mag) {
  if constexpr (KIND == KIND_E4M3 && EPI == EPI_DGRAD) return e4m3_mag_bits(e4m3_from_f32(__uint_as_float(mag)));
  else if constexpr (KIND == KIND_F16) return mag_bits(f16_to_f32(f16_from_f32(__uint_as_float(mag))));
  else return mag;
}

// Direct (non-TMA) store of one unit: used when the output rows are not
// 16-byte aligned or when accumulating into the existing gradient.
__device__ __forceinline__ void store_unit_direct(const EpiArgs& ea, int row, int col0, int nv, uint32_t (&r)[64],
                                                  bool out16) {
  if (out16) {
    uint16_t* o = static_cast<uint16_t*>(ea.out) + (int64_t)row * ea.ldo + col0;
    if (nv >= 64 && ea.vec_out) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<uint4*>(o)[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j < nv) o[j] = (uint16_t)((r[j >> 1] >> (16 * (j & 1))) & 0xFFFFu);
    }
  } else {
    float* o = static_cast<float*>(ea.out) + (int64_t)row * ea.ldo + col0;
    if (ea.accumulate) {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j < nv) r[j] = __float_as_uint(o[j] + fu(r[j]));
    }
    if (nv >= 64 && ea.vec_out) {
#pragma unroll
      for (int q = 0; q < 16; ++q)
        reinterpret_cast<uint4*>(o)[q] = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j < nv) o[j] = fu(r[j]);
    }
  }
}

// Stage 32 words (128 bytes) of this lane's row into the warp's 4 KB buffer
// in the 128-byte-swizzled layout the output tensor map expects (16-byte
// chunk c of row r lands at chunk c ^ (r % 8)): conflict-free stores.
__device__ __forceinline__ void stage_row(uint8_t* buf, int lane, const uint32_t* w) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) =
        make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Store one 32-row x 128-byte box from registers (lane = row, w[0..31] = the
// row's 32 words) without the TMA unit: stage the rows in the warp's buffer
// (swizzled, conflict-free), read them back so that lane l holds 16-byte
// chunk l%8 of row 4i + l/8, and store: every warp instruction then writes
// four full 128-byte rows. The buffer is free again when this returns.
// accumulate: add the existing fp32 values (read the same way).
__device__ __forceinline__ void store_box_coalesced(const EpiArgs& ea, uint8_t* buf, int lane, const uint32_t* w,
                                                    int row0, int x, int es) {
  stage_row(buf, lane, w);
  __syncwarp();
  const int c = lane & 7;
  const int per = 16 / es;   // elements per chunk
  const int col = x + c * per;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    uint4 v = *reinterpret_cast<const uint4*>(buf + r * 128 + ((c ^ (r & 7)) << 4));
    const int grow = row0 + r;
    if (grow < ea.M && col < ea.N) {
      uint8_t* dst = static_cast<uint8_t*>(ea.out) + ((int64_t)grow * ea.ldo + col) * es;
      if (col + per <= ea.N) {
        if (ea.accumulate) {
          const float4 o = *reinterpret_cast<const float4*>(dst);
          v.x = __float_as_uint(o.x + fu(v.x));
          v.y = __float_as_uint(o.y + fu(v.y));
          v.z = __float_as_uint(o.z + fu(v.z));
          v.w = __float_as_uint(o.w + fu(v.w));
        }
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
        for (int e = 0; e < per && col + e < ea.N; ++e) {
          if (es == 4) {
            float* d = reinterpret_cast<float*>(dst) + e;
            *d = ea.accumulate ? *d + fu(vw[e]) : fu(vw[e]);
          } else {
            reinterpret_cast<uint16_t*>(dst)[e] = (uint16_t)(vw[e >> 1] >> (16 * (e & 1)));
          }
        }
      }
    }
  }
  __syncwarp();
}

// Tile order: groups of kGroupM consecutive M blocks, N advancing across a
// group and M fastest inside it, so the CTAs running at the same time share
// their B tiles (and a group's A rows) in L2 even when B is larger than L2
// (e.g. a 50k-row vocabulary projection).
constexpr int kGroupM = 16;

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group, int& m_blk, int& n_blk) {
  const int group_tiles = group * num_n;
  const int g = tile / group_tiles;
  const int first_m = g * group;
  const int gs = min(group, num_m - first_m);
  const int local = tile - g * group_tiles;
  m_blk = first_m + local % gs;
  n_blk = local / gs;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <int KIND, int BN, int EPI, bool PAIR, int EW>
__global__ void __launch_bounds__(threads_for<EW>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmO, EpiArgs ea) {
  using C = Cfg<BN, PAIR, EW>;
  constexpr int kEpiWarps = C::kEpiWarps;
  constexpr int kEpiThreads = C::kEpiThreads;
  constexpr int kStages = C::kStages;
  constexpr int kElemPerSlab = kSlab / KindInfo<KIND>::bytes;
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* smA = smem;
  uint8_t* smB = smem + kStages * C::kABytes;
  uint8_t* sEpi = smem + kStages * C::kStageBytes;                 // per warp: kEpiBufs x 4 KB staging
  float* sBias = reinterpret_cast<float*>(sEpi + kEpiWarps * C::kEpiBufs * kEpiStageBytes);   // per warp: its columns
  uint64_t* full = reinterpret_cast<uint64_t*>(sBias + kEpiWarps * C::kWarpCols);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // PAIR: clusters of two CTAs; rank 0 (the even CTA) issues the MMAs
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr int kGroup = PAIR ? kGroupM / 2 : kGroupM;
  const int num_n = (ea.N + BN - 1) / BN;
  const int num_m = (ea.M + C::kTileM - 1) / C::kTileM;
  const int num_tiles = num_m * num_n;
  const int kb_count = (int)(((int64_t)ea.K * KindInfo<KIND>::bytes + kSlab - 1) / kSlab);
  // work units: (tile, K range)
  const int num_units = num_work_units(ea, num_tiles);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps * C::kCtas);   // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"((uint32_t)C::kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"((uint32_t)C::kTmemCols)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  fence_before();
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the previous kernel's outputs (operands, counters, workspace) are ready
  pdl_wait();
  // data parallel: this launch's place in the gradient's sequence of averages
  const unsigned int dp_epoch = (EPI == EPI_WGRAD && ea.dp.mc != nullptr) ? *ea.dp.epoch : 0u;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = unit0; ok && w < num_units; w += units) {
        const Unit un = unit_of(ea, w, kb_count);
        const int kb0 = un.kb0, kb1 = un.kb1;
        int m_blk, n_blk;
        tile_coords(un.tile, num_m, num_n, kGroup, m_blk, n_blk);
        const int a_row = m_blk * C::kTileM + (int)rank * BM;
        const int b_row = n_blk * BN + (int)rank * C::kBRows;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, kStatusTimeoutEmpty)) { ok = false; break; }
          if constexpr (PAIR) {
            // the even CTA's full barrier expects both CTAs' bytes
            if (rank == 0) mbar_expect_tx(&full[stage], C::kCtas * C::kStageBytes);
            const uint32_t bar = map_to_cta(&full[stage], 0);
            tma_load_2d_pair(smA + stage * C::kABytes, &tmA, kb * kElemPerSlab, a_row, bar);
            tma_load_2d_pair(smB + stage * C::kBBytes, &tmB, kb * kElemPerSlab, b_row, bar);
          } else {
            mbar_expect_tx(&full[stage], C::kStageBytes);
            tma_load_2d(smA + stage * C::kABytes, &tmA, kb * kElemPerSlab, a_row, &full[stage]);
            tma_load_2d(smB + stage * C::kBBytes, &tmB, kb * kElemPerSlab, b_row, &full[stage]);
          }
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
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      constexpr uint32_t id = idesc<KIND, BN, C::kTileM>();
      for (int w = unit0; ok && w < num_units; w += units, ++local) {
        const Unit un = unit_of(ea, w, kb_count);
        const int kb0 = un.kb0, kb1 = un.kb1;
        const int acc = local & 1;
        const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
        if (!mbar_wait<PAIR>(&tempty[acc], acc_par ^ 1u, kStatusTimeoutAcc)) { ok = false; break; }
        fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, kStatusTimeoutFull)) { ok = false; break; }
          fence_after();
          const uint32_t a0 = smem_u32(smA + stage * C::kABytes);
          const uint32_t b0 = smem_u32(smB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < kSlab / 32; ++k)
            mma<KIND, PAIR>(d, sdesc(a0 + 32 * k), sdesc(b0 + 32 * k), id, (kb != kb0 || k != 0) ? 1u : 0u);
          mma_commit<PAIR>(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) mma_commit<PAIR>(&tfull[acc]);
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2 .. 2+kEpiWarps-1: TMEM lane quarter warp%4, column
    // part (warp-2)/4 of the tile
    const int q = warp & 3;
    const int e = warp - 2;
    const int part = e >> 2;
    constexpr int kUnits = C::kWarpCols / 64;                // 64-column units per warp
    uint8_t* stage_base = sEpi + e * C::kEpiBufs * kEpiStageBytes;
    float* sb = sBias + e * C::kWarpCols;
    const bool out16 = ea.out_dt != APA_DT_F32;
    EpiState st;
    int local = 0;
    int slot = 0, inflight = 0;   // staging ring position, stores not yet known to be read
    // accumulator hand-back: one arrival per warp on the MMA CTA's barrier
    const uint32_t tempty0 = PAIR ? map_to_cta(&tempty[0], 0) : 0u;
    const uint32_t tempty1 = PAIR ? map_to_cta(&tempty[1], 0) : 0u;
    auto release_acc = [&](int acc) {
      fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(acc ? tempty1 : tempty0);
        else mbar_arrive(&tempty[acc]);
      }
    };
    // forward bias: the first tile's columns now, each later tile's during
    // the tile before it
    BiasRaw<C::kWarpCols> braw;
    auto bias_cols = [&](int w) {
      int mb, nb;
      tile_coords(unit_of(ea, w, kb_count).tile, num_m, num_n, kGroup, mb, nb);
      return nb * BN + part * C::kWarpCols;
    };
    if constexpr (EPI == EPI_FWD) {
      if (ea.bias != nullptr && unit0 < num_units) bias_load<KIND, C::kWarpCols>(ea, bias_cols(unit0), lane, braw);
    }
    for (int w = unit0; w < num_units; w += units, ++local) {
      const Unit un = unit_of(ea, w, kb_count);
      const int tile = un.tile;
      const int orow_off = un.orow;   // this split's slice of the output (split-K)
      const int acc = local & 1;
      const uint32_t acc_par = (uint32_t)(local >> 1) & 1u;
      int m_blk, n_blk;
      tile_coords(tile, num_m, num_n, kGroup, m_blk, n_blk);
      const int col_base = n_blk * BN + part * C::kWarpCols;   // this warp's first column
      const int row0 = m_blk * C::kTileM + (int)rank * BM + q * 32;
      const int row = row0 + lane;
      const bool row_ok = row < ea.M;
      const bool check = (row0 + 32 > ea.M) || (col_base + C::kWarpCols > ea.N);
      if constexpr (EPI == EPI_FWD) {
        if (ea.bias != nullptr) {
          __syncwarp();   // every lane is done with the previous tile's row
          bias_store<KIND, C::kWarpCols>(sb, lane, braw);
          __syncwarp();
          if (w + units < num_units) bias_load<KIND, C::kWarpCols>(ea, bias_cols(w + units), lane, braw);
        }
      }
      // one lane waits and the warp follows its verdict, so a timeout can
      // never split the warp ahead of the warp-collective TMEM loads
      bool ready = true;
      if (lane == 0) ready = mbar_wait(&tfull[acc], acc_par, kStatusTimeoutAcc);
      ready = __shfl_sync(0xFFFFFFFFu, ready ? 1 : 0, 0) != 0;
      if (!ready) break;
      fence_after();
      const uint32_t tbase =
          tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN) + (uint32_t)(part * C::kWarpCols);
      bool released = false;
      // stream-K tail unit (two splits): store this split's raw partial
      // (lane-major, so each warp store writes 512 contiguous bytes), then
      // take the ticket of this warp's part of the tile; the warp that takes
      // the second ticket adds the other split's partial to its own and runs
      // the epilogue. fp32 addition commutes, so the sum has the same bits
      // whichever split finishes last.
      const float4* sk_other = nullptr;   // set: this warp finishes the tile
      if (un.sk_split >= 0) {
        constexpr int kChunk4 = C::kWarpCols * 8;   // float4s per warp and split (kWarpCols x 32 lanes / 4)
        const int tail = tile - ea.sk_first;
        const int64_t widx = (int64_t)rank * kEpiWarps + e;
        const int64_t per_split = (int64_t)C::kCtas * kEpiWarps;
        float4* mine = reinterpret_cast<float4*>(ea.sk_ws) +
                       (((int64_t)tail * 2 + un.sk_split) * per_split + widx) * kChunk4 + lane;
#pragma unroll 1
        for (int u = 0; u < kUnits; ++u) {
          if (col_base + u * 64 >= ea.N) break;   // warp-uniform
          uint32_t r[64];
          tmem_ld32_nowait(tbase + (uint32_t)(u * 64), r);
          tmem_ld32_nowait(tbase + (uint32_t)(u * 64 + 32), r + 32);
          tmem_wait_ld();
#pragma unroll
          for (int c4 = 0; c4 < 16; ++c4)
            mine[(u * 16 + c4) * 32] = make_float4(fu(r[4 * c4]), fu(r[4 * c4 + 1]), fu(r[4 * c4 + 2]),
                                                   fu(r[4 * c4 + 3]));
        }
        __threadfence();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(&ea.sk_tickets[(int64_t)tail * per_split + widx], 1);
        old = __shfl_sync(0xFFFFFFFFu, old, 0);
        if (old == 0) {
          release_acc(acc);   // the other split's warp finishes this part of the tile
          continue;
        }
        __threadfence();
        sk_other = reinterpret_cast<const float4*>(ea.sk_ws) +
                   (((int64_t)tail * 2 + (1 - un.sk_split)) * per_split + widx) * kChunk4 + lane;
      }
#pragma unroll 1
      for (int u = 0; u < kUnits; ++u) {
        const int col0 = col_base + u * 64;
        if (col0 >= ea.N) break;   // warp-uniform
        const int nv = min(64, ea.N - col0);
        uint32_t r[64];
        tmem_ld32_nowait(tbase + (uint32_t)(u * 64), r);
        tmem_ld32_nowait(tbase + (uint32_t)(u * 64 + 32), r + 32);
        tmem_wait_ld();
        if (u == kUnits - 1 || col0 + 64 >= ea.N) {
          // every TMEM read of this warp's part of the accumulator is done
          release_acc(acc);
          released = true;
        }
        if (sk_other != nullptr) {
#pragma unroll
          for (int c4 = 0; c4 < 16; ++c4) {
            const float4 v = __ldcg(sk_other + (u * 16 + c4) * 32);
            r[4 * c4] = __float_as_uint(fu(r[4 * c4]) + v.x);
            r[4 * c4 + 1] = __float_as_uint(fu(r[4 * c4 + 1]) + v.y);
            r[4 * c4 + 2] = __float_as_uint(fu(r[4 * c4 + 2]) + v.z);
            r[4 * c4 + 3] = __float_as_uint(fu(r[4 * c4 + 3]) + v.w);
          }
        }
        epi_unit<KIND, EPI>(ea, sb + u * 64, r, st, check, row_ok, nv);
        if (ea.coalesced_out) {
          if (row0 < ea.M) {
            const int nbox = out16 ? 1 : 2;
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              const int x = col0 + b * 32;
              if (b >= nbox || x >= ea.N) break;
              store_box_coalesced(ea, stage_base, lane, r + 32 * b, row0, out16 ? col0 : x, out16 ? 2 : 4);
            }
          }
        } else if (ea.tma_out) {
          if (row0 < ea.M) {
            const int nbox = out16 ? 1 : 2;
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              const int x = col0 + b * 32;
              if (b >= nbox || x >= ea.N) break;
              if (inflight >= C::kEpiBufs) {
                // the store that last used this slot must have read it
                if (lane == 0) bulk_wait_read<C::kEpiBufs - 1>();
                __syncwarp();
                inflight = C::kEpiBufs - 1;
              }
              uint8_t* buf = stage_base + slot * kEpiStageBytes;
              stage_row(buf, lane, r + 32 * b);
              fence_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmO, buf, x, row0 + orow_off);
                bulk_commit();
              }
              ++inflight;
              slot = slot + 1 == C::kEpiBufs ? 0 : slot + 1;
            }
          }
        } else if (row_ok) {
          store_unit_direct(ea, row + orow_off, col0, nv, r, out16);
        }
      }
      if (!released) release_acc(acc);   // this warp's columns lie past N: keep the count exact
      if constexpr (EPI == EPI_WGRAD) {
        if (ea.dp.mc != nullptr && row0 < ea.M) {
          // data parallel: this warp's part of the tile is stored (TMA stores
          // complete, direct stores fenced); publish its regions to every
          // rank, then average the ones this rank owns while the tensor
          // cores work on the next tiles
          if (lane == 0 && inflight > 0) bulk_wait_all();
          inflight = 0;
          asm volatile("fence.proxy.async.global;" ::: "memory");
          dpr::fence_sys();
          __syncwarp();
          const int rb = row0 / dpr::kRegionRows;
          const int ncb = dpr::region_cols(ea.N);
          if (lane == 0) {
            for (int u = 0; u < kUnits; ++u) {
              const int col0 = col_base + u * 64;
              if (col0 >= ea.N) break;
              dpr::signal_ready(ea.dp, (int64_t)rb * ncb + col0 / dpr::kRegionCols);
            }
          }
          for (int u = 0; u < kUnits; ++u) {
            const int col0 = col_base + u * 64;
            if (col0 >= ea.N) break;
            const int64_t g = (int64_t)rb * ncb + col0 / dpr::kRegionCols;
            if ((int)(g % ea.dp.world) == ea.dp.rank)
              dpr::reduce_region(ea.dp, rb, col0 / dpr::kRegionCols, dp_epoch, lane);
          }
        }
      }
    }
    const bool pending_store = inflight > 0;
    if (pending_store && lane == 0) bulk_wait_all();
    __syncwarp();
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
      if (lane == 0 && m != 0u) telem_commit(ea.amax, ea.flag, final_mag<KIND, EPI>(m));
    }
    if constexpr (EPI == EPI_WGRAD) {
      // named barrier over the epilogue warps, then one ticket per CTA
      asm volatile("bar.sync 1, %0;" ::"r"(kEpiThreads) : "memory");
      if (threadIdx.x == 64 && ea.counters) {
        __threadfence();
        const unsigned long long ticket = atomicAdd(&ea.counters[2], 1ull);
        if (ticket == (unsigned long long)gridDim.x - 1ull) {
          __threadfence();
          if (ea.finalize) {
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
          }
          ea.counters[2] = 0ull;
        }
      }
    }
  }

  // PAIR: neither CTA leaves (or frees TMEM) while the other may still signal
  // its barriers or read its accumulators
  fence_before();
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  fence_after();
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"((uint32_t)C::kTmemCols)
                   : "memory");
    } else {
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"((uint32_t)C::kTmemCols)
                   : "memory");
    }
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

// Output map for the epilogue's TMA stores: dims {N (inner), M}, row pitch
// ldo elements, box {128 bytes, 32 rows}, 128-byte swizzle (the staging
// layout). Returns false when the output cannot be stored this way.
bool make_out_map(CUtensorMap* tm, const EpiArgs& ea) {
  EncodeFn enc = get_encode();
  if (!enc || ea.accumulate) return false;
  int es;
  CUtensorMapDataType dt;
  switch (ea.out_dt) {
    case APA_DT_F32: es = 4; dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    case APA_DT_F16: es = 2; dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case APA_DT_BF16: es = 2; dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    default: return false;
  }
  if ((reinterpret_cast<uintptr_t>(ea.out) & 15u) != 0 || ((ea.ldo * es) & 15) != 0) return false;
  // split-K: the stacked slices, each split_rows long
  const int64_t rows = ea.splits > 1 ? (int64_t)ea.split_rows * ea.splits : (int64_t)ea.M;
  cuuint64_t dims[2] = {(cuuint64_t)ea.N, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ea.ldo * es)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), 32u};
  cuuint32_t estr[2] = {1, 1};
  return enc(tm, dt, 2, ea.out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Number of two-CTA clusters of this kernel that fit on the device at once
// (0 when none does), computed once per kernel.
template <int KIND, int BN, int EPI, int EW>
int pair_capacity() {
  using C = Cfg<BN, true, EW>;
  static std::once_flag once;
  static int clusters = 0;
  std::call_once(once, [] {
    if (cudaFuncSetAttribute(gemm_kernel<KIND, BN, EPI, true, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemBytes) != cudaSuccess)
      return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms(), 1, 1);
    cfg.blockDim = dim3(C::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<KIND, BN, EPI, true, EW>, &cfg) == cudaSuccess) clusters = n;
    else (void)cudaGetLastError();
  });
  return clusters;
}

// Stream-K split of the last, partial wave: with `tiles` tiles on `slots`
// CTAs (or CTA pairs), W full waves and R < slots left over, the R tail
// tiles are each split along K into two units (at least 8 slabs each) that
// run side by side, so the tail costs about half a tile instead of a whole
// one. Only when the tail fills at most half a wave. Workspace: 2 R fp32 tile
// partials, then one int ticket per tail tile, CTA and epilogue warp.
struct TailPlan {
  int first, splits, kb_per_split;
  int64_t part_bytes, bytes;
};

inline TailPlan tail_plan(int64_t tiles, int64_t slots, int64_t kb_count, int64_t tile_elems, int ctas_x_warps) {
  TailPlan t{0, 0, 0, 0, 0};
  if (slots < 2 || tiles < slots) return t;
  const int64_t W = tiles / slots, R = tiles - W * slots;
  if (R == 0 || 2 * R > slots) return t;
  if (kb_count < 16) return t;
  const int64_t S = 2;
  const int64_t per = (kb_count + 1) / 2;
  t.first = (int)(W * slots);
  t.splits = (int)S;
  t.kb_per_split = (int)per;
  t.part_bytes = R * S * tile_elems * 4;
  t.bytes = t.part_bytes + (R * ctas_x_warps * 4 + 15) / 16 * 16;
  return t;
}

template <int BN, bool PAIR, int EW>
TailPlan tail_plan_for(const EpiArgs& ea, int kind_bytes, int64_t slots) {
  using C = Cfg<BN, PAIR, EW>;
  const int64_t tiles = ((int64_t)(ea.M + C::kTileM - 1) / C::kTileM) * ((ea.N + BN - 1) / BN);
  const int64_t kb_count = ((int64_t)ea.K * kind_bytes + kSlab - 1) / kSlab;
  return tail_plan(tiles, slots, kb_count, (int64_t)C::kTileM * BN, C::kCtas * EW);
}

template <int KIND, int BN, int EPI, bool PAIR, int EW>
int launch_t(const void* A, int64_t lda, const void* B, int64_t ldb, EpiArgs ea, int grid_cap, cudaStream_t s) {
  using C = Cfg<BN, PAIR, EW>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(gemm_kernel<KIND, BN, EPI, PAIR, EW>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  });
  if (attr_err != cudaSuccess) return APA_ERR_CUDA;
  CUtensorMap ta, tb;
  int st = make_map(&ta, KIND, A, ea.M, ea.K, lda, BM);
  if (st) return st;
  st = make_map(&tb, KIND, B, ea.N, ea.K, ldb, C::kBRows);
  if (st) return st;
  CUtensorMap to = ta;
  // aligned outputs: TMA bulk-tensor stores (measured faster than coalesced
  // st.global from the same staging); accumulating into an aligned fp32
  // gradient: coalesced read-add-store through the staging buffer
  ea.tma_out = make_out_map(&to, ea) ? 1 : 0;
  ea.coalesced_out = (!ea.tma_out && ea.accumulate && ea.vec_out) ? 1 : 0;
  // work units: tiles x K splits
  int tiles = ((ea.M + C::kTileM - 1) / C::kTileM) * ((ea.N + BN - 1) / BN) * (ea.splits > 1 ? ea.splits : 1);
  // stream-K tail (caller workspace given, no split-K): planned against the
  // number of CTAs (pairs) that actually run
  auto plan_tail = [&](int64_t slots) -> int {
    ea.sk_splits = 0;
    if (ea.sk_ws == nullptr || ea.splits > 1) return APA_OK;
    const TailPlan tp = tail_plan_for<BN, PAIR, EW>(ea, KindInfo<KIND>::bytes, slots);
    if (tp.splits < 2 || tp.bytes > ea.sk_ws_bytes) return APA_OK;
    ea.sk_first = tp.first;
    ea.sk_splits = tp.splits;
    ea.sk_kb_per_split = tp.kb_per_split;
    ea.sk_tickets = reinterpret_cast<int*>(reinterpret_cast<char*>(ea.sk_ws) + tp.part_bytes);
    if (cudaMemsetAsync(ea.sk_tickets, 0, (size_t)(tp.bytes - tp.part_bytes), s) != cudaSuccess) return APA_ERR_CUDA;
    tiles = num_work_units(ea, tiles);
    return APA_OK;
  };
  if constexpr (PAIR) {
    const int cap = pair_capacity<KIND, BN, EPI, EW>();
    if (cap < 1) return APA_ERR_UNSUPPORTED;
    const int slots = std::max(1, std::min(grid_cap > 0 ? std::max(1, grid_cap / 2) : cap, cap));
    if (int st = plan_tail(slots)) return st;
    int clusters = std::min(tiles, slots);
    clusters = std::max(1, clusters);
    if (launch_kernel(gemm_kernel<KIND, BN, EPI, true, EW>, dim3(2 * clusters), dim3(C::kThreads), C::kSmemBytes,
                      s, 2, ta, tb, to, ea) != cudaSuccess)
      return APA_ERR_CUDA;
  } else {
    const int slots = std::max(1, grid_cap > 0 ? grid_cap : num_sms());
    if (int st = plan_tail(slots)) return st;
    int grid = std::min(tiles, slots);
    if (grid < 1) grid = 1;
    if (launch_kernel(gemm_kernel<KIND, BN, EPI, false, EW>, dim3(grid), dim3(C::kThreads), C::kSmemBytes, s, 1,
                      ta, tb, to, ea) != cudaSuccess)
      return APA_ERR_CUDA;
  }
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

// Tile shapes: 128 x 128 and 128 x 256 on one CTA, 256 x 256 on a CTA pair;
// flag bits select the epilogue width (0 = automatic).
constexpr int kTile128 = 128, kTile256 = 256, kTilePair = 512;
constexpr int kEpiFlag4 = 1, kEpiFlag8 = 2;

template <int KIND, int EPI, int EW>
int launch_shape(const void* A, int64_t lda, const void* B, int64_t ldb, EpiArgs ea, int tile, int grid_cap,
                 cudaStream_t s) {
  if (tile == kTilePair) return launch_t<KIND, 256, EPI, true, EW>(A, lda, B, ldb, ea, grid_cap, s);
  if (tile == kTile256) return launch_t<KIND, 256, EPI, false, EW>(A, lda, B, ldb, ea, grid_cap, s);
  return launch_t<KIND, 128, EPI, false, EW>(A, lda, B, ldb, ea, grid_cap, s);
}

template <int KIND, int EPI>
int launch_bn(const void* A, int64_t lda, const void* B, int64_t ldb, EpiArgs ea, int tile, int ew, int grid_cap,
              cudaStream_t s) {
  if (ew == 8) return launch_shape<KIND, EPI, 8>(A, lda, B, ldb, ea, tile, grid_cap, s);
  return launch_shape<KIND, EPI, 4>(A, lda, B, ldb, ea, tile, grid_cap, s);
}

// Split-K phase 2 for a weight gradient: sum the fp32 partial slices in
// split order (deterministic), then exactly the weight-gradient epilogue of
// the GEMM: counts of nonzero / underflow values (on the fp32 sum; at FP16 on
// its fp16 rounding), the rounding to the working dtype and the fp32 store
// (or accumulate), and the last block's ratio fold into the running max.
template <int KIND, bool VEC>
__global__ void __launch_bounds__(256) wgrad_reduce_kernel(const float* ws, int splits, int64_t slice, int64_t ld_ws,
                                                           int rows, int cols, float* dw, int64_t lddw, int accumulate,
                                                           float vmin, unsigned long long* counters,
                                                           float* ratio_max) {
  // VEC: four adjacent columns per thread (cols, ld_ws and lddw multiples of
  // 4, dw 16-byte aligned); rows * cols < 2^31 (the split path only takes
  // small gradients)
  constexpr int V = VEC ? 4 : 1;
  pdl_launch_dependents();
  pdl_wait();
  __shared__ unsigned int s_nz[8], s_uf[8];
  const uint32_t vb = __float_as_uint(vmin);
  unsigned int nz = 0, uf = 0;
  const uint32_t cq = (uint32_t)(cols / V);
  const uint32_t total = (uint32_t)rows * cq;
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
    const uint32_t r = e / cq, c = (e - r * cq) * V;
    const float* src = ws + (int64_t)r * ld_ws + c;
    float acc[V];
    if constexpr (VEC) {
      const float4 v = *reinterpret_cast<const float4*>(src);
      acc[0] = v.x; acc[1] = v.y; acc[2] = v.z; acc[3] = v.w;
    } else {
      acc[0] = src[0];
    }
    // at most 8 splits: every split's load is issued before the adds, which
    // run in split order
#pragma unroll
    for (int sp = 1; sp < 8; ++sp) {
      if (sp < splits) {
        if constexpr (VEC) {
          const float4 v = *reinterpret_cast<const float4*>(src + sp * slice);
          acc[0] += v.x; acc[1] += v.y; acc[2] += v.z; acc[3] += v.w;
        } else {
          acc[0] += src[sp * slice];
        }
      }
    }
    float res[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float out;
      if constexpr (KIND == KIND_E4M3) {
        const uint32_t a = (__float_as_uint(acc[i]) & 0x7FFFFFFFu) - 1u;
        nz += a < 0x7F800000u ? 1u : 0u;
        uf += a < vb - 1u ? 1u : 0u;
        out = e4m3_to_f32(e4m3_from_f32(acc[i]));
      } else if constexpr (KIND == KIND_F16) {
        out = f16_to_f32(f16_from_f32(acc[i]));
        const uint32_t a = (__float_as_uint(out) & 0x7FFFFFFFu) - 1u;
        nz += a < 0x7F800000u ? 1u : 0u;
        uf += a < vb - 1u ? 1u : 0u;
      } else {
        out = acc[i];
      }
      res[i] = out;
    }
    float* d = dw + (int64_t)r * lddw + c;
    if constexpr (VEC) {
      float4 o = make_float4(res[0], res[1], res[2], res[3]);
      if (accumulate) {
        const float4 old = *reinterpret_cast<const float4*>(d);
        o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
      }
      *reinterpret_cast<float4*>(d) = o;
    } else {
      *d = accumulate ? *d + res[0] : res[0];
    }
  }
  if (!counters) return;
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
      const unsigned long long nzc = atomicAdd(&counters[0], 0ull);
      const unsigned long long ufc = atomicAdd(&counters[1], 0ull);
      float ratio = 0.0f;
      if (nzc != 0ull) ratio = __fdiv_rn(__ull2float_rn(ufc), __ull2float_rn(nzc));
      if (ratio_max) {
        const float old = *ratio_max;
        *ratio_max = (old != old) ? old : fmaxf(old, ratio);
      }
      counters[0] = 0ull;
      counters[1] = 0ull;
      counters[2] = 0ull;
    }
  }
}

template <int KIND, int EPI>
bool pair_ok() {
  return pair_capacity<KIND, 256, EPI, 4>() > 0 && pair_capacity<KIND, 256, EPI, 8>() > 0;
}

}  // namespace gemm

// Upper bound on the persistent grid (0 = one CTA per SM). Set while a
// collective runs concurrently, so its kernel finds free SMs.
static int g_gemm_sm_limit = 0;

struct GemmPlan {
  int tile, ew;
};

// Tile shape and epilogue width from an estimate of the persistent
// schedule's length: waves (work units over the CTAs or pairs that run at
// once) times the cost of one unit. Two regimes:
//  * epilogue-bound (few 128-byte K slabs per tile for the bytes each output
//    element stores): a unit costs its valid output columns; a 128-wide unit
//    0.55 of a 256-wide one (half the outputs plus fixed per-tile work); a
//    CTA pair gains nothing;
//  * mainloop-bound: a 128-wide unit costs 0.7 of a 256-wide one (it reads more
//    operand bytes per output); a CTA pair reads 1.5x fewer operand bytes than
//    two single CTAs, worth ~8 % once each pair runs three or more tiles or
//    one long reduction (512 or more 128-byte K slabs: 7 % measured on a TF32
//    8192 x 1024 x 50304 input gradient); in one or two short waves the
//    cluster's lock-step loads cost as much.
// Eight epilogue warps for epilogue-bound shapes; otherwise four warps and a
// deeper operand pipeline, also when each CTA runs only one or two tiles
// (measured on 8192 x 1024 x 4096: FP8 forward 31.5 against 35.0 µs, FP16
// input gradient 67 against 76 µs).
GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int es, int out_es, int slots, bool pair_possible, int tile,
                   int epi) {
  using namespace gemm;
  auto cdiv = [](int64_t a, int64_t b) { return (a + b - 1) / b; };
  const int64_t sms = std::max(1, slots);
  const int64_t k_bytes = K * es;
  const bool epi_bound = k_bytes * 4 <= 2048 * (int64_t)out_es;
  auto width = [&](int bn) { return epi_bound ? (double)N / (double)(cdiv(N, bn) * bn) : 1.0; };
  const int64_t tiles128 = cdiv(M, 128) * cdiv(N, 128);
  const int64_t tiles256 = cdiv(M, 128) * cdiv(N, 256);
  const int64_t tilesP = cdiv(M, 256) * cdiv(N, 256);
  const int64_t pairs = std::max<int64_t>(1, sms / 2);
  if (tile != kTile128 && tile != kTile256 && tile != kTilePair) {
    const double t128 = (double)cdiv(tiles128, sms) * width(128) * (epi_bound ? 0.55 : 0.7);
    const double t256 = (double)cdiv(tiles256, sms) * width(256);
    double best = t256;
    tile = kTile256;
    if (t128 < best) { best = t128; tile = kTile128; }
    if (pair_possible && M > 128) {
      const int64_t w = cdiv(tilesP, pairs);
      const bool long_k = k_bytes >= 512 * (int64_t)kSlab;
      // an epilogue-bound forward GEMM (fp32 output, telemetry) measured
      // 10-12 % faster on the pair with eight epilogue warps at equal wave
      // counts (8192 tokens x 1024 -> 3072 / 4096: 35.8 against 40.8 µs,
      // 41.5 against 47.1 µs); epilogue-bound input gradients did not
      const double gain = (!epi_bound && (w >= 3 || long_k)) ? 1.0 / 1.08
                          : (epi_bound && epi == EPI_FWD) ? 0.9 : 1.0 / 0.97;
      const double tp = (double)w * width(256) * gain;
      if (tp < best) { best = tp; tile = kTilePair; }
    }
  }
  const int ew = epi_bound ? 8 : 4;
  return {tile, ew};
}

// Whether the CTA-pair kernels of this rung / epilogue can run on the device.
bool pair_possible(int rung, int epi) {
  using namespace gemm;
#define APA_PAIR_CASE(KIND)                                  \
  switch (epi) {                                             \
    case EPI_FWD: return pair_ok<KIND, EPI_FWD>();           \
    case EPI_DGRAD: return pair_ok<KIND, EPI_DGRAD>();       \
    case EPI_WGRAD: return pair_ok<KIND, EPI_WGRAD>();       \
    case EPI_RAW: return pair_ok<KIND, EPI_RAW>();           \
    default: return false;                                   \
  }
  switch (rung) {
    case APA_RUNG_FP8: APA_PAIR_CASE(KIND_E4M3)
    case APA_RUNG_FP16: APA_PAIR_CASE(KIND_F16)
    case APA_RUNG_TF32: APA_PAIR_CASE(KIND_TF32)
    default: return false;
  }
#undef APA_PAIR_CASE
}

// The launch configuration of one GEMM: tile code (possibly with epilogue
// flag bits) and grid cap resolved exactly as gemm_dispatch resolves them.
int resolve_plan(int rung, int epi, int64_t M, int64_t N, int64_t K, int out_dt, int tile, int grid_cap,
                 GemmPlan* out) {
  using namespace gemm;
  if (rung != APA_RUNG_FP8 && rung != APA_RUNG_FP16 && rung != APA_RUNG_TF32) return APA_ERR_INVALID;
  if (epi != EPI_FWD && epi != EPI_DGRAD && epi != EPI_WGRAD && epi != EPI_RAW) return APA_ERR_INVALID;
  if (grid_cap <= 0 && g_gemm_sm_limit > 0) grid_cap = g_gemm_sm_limit;
  const int ew_flag = tile & 3;
  tile &= ~3;
  const bool pair = pair_possible(rung, epi);
  if (tile == kTilePair && !pair) return APA_ERR_UNSUPPORTED;
  const int es = rung == APA_RUNG_FP8 ? 1 : rung == APA_RUNG_FP16 ? 2 : 4;
  const int out_es = out_dt == APA_DT_F32 ? 4 : 2;
  GemmPlan pl = plan_gemm(M, N, K, es, out_es, grid_cap > 0 ? grid_cap : num_sms(), pair, tile, epi);
  if (ew_flag == kEpiFlag4) pl.ew = 4;
  if (ew_flag == kEpiFlag8) pl.ew = 8;
  *out = pl;
  return APA_OK;
}

int gemm_dispatch(int rung, int epi, const void* A, int64_t lda, const void* B, int64_t ldb, gemm::EpiArgs ea,
                  int tile, int grid_cap, cudaStream_t s) {
  using namespace gemm;
  GemmPlan pl;
  if (int st = resolve_plan(rung, epi, ea.M, ea.N, ea.K, ea.out_dt, tile, grid_cap, &pl)) return st;
  if (grid_cap <= 0 && g_gemm_sm_limit > 0) grid_cap = g_gemm_sm_limit;
#define APA_EPI_CASE(KIND)                                                                                \
  switch (epi) {                                                                                           \
    case EPI_FWD: return launch_bn<KIND, EPI_FWD>(A, lda, B, ldb, ea, pl.tile, pl.ew, grid_cap, s);        \
    case EPI_DGRAD: return launch_bn<KIND, EPI_DGRAD>(A, lda, B, ldb, ea, pl.tile, pl.ew, grid_cap, s);    \
    case EPI_RAW: return launch_bn<KIND, EPI_RAW>(A, lda, B, ldb, ea, pl.tile, pl.ew, grid_cap, s);        \
    default: return launch_bn<KIND, EPI_WGRAD>(A, lda, B, ldb, ea, pl.tile, pl.ew, grid_cap, s);           \
  }
  switch (rung) {
    case APA_RUNG_FP8: APA_EPI_CASE(KIND_E4M3)
    case APA_RUNG_FP16: APA_EPI_CASE(KIND_F16)
    default: APA_EPI_CASE(KIND_TF32)
  }
#undef APA_EPI_CASE
}

// Clusters of the pair kernel that fit on the device.
template <int KIND, int EPI>
int cap_of(int ew) {
  using namespace gemm;
  return ew == 8 ? pair_capacity<KIND, 256, EPI, 8>() : pair_capacity<KIND, 256, EPI, 4>();
}

// Workspace the stream-K tail of this GEMM would use with the launch
// configuration gemm_dispatch picks now (0 when the last wave is full or
// more than half full).
int tail_workspace_bytes(int rung, int epi, const gemm::EpiArgs& ea, int64_t* bytes_out) {
  using namespace gemm;
  *bytes_out = 0;
  GemmPlan pl;
  if (int st = resolve_plan(rung, epi, ea.M, ea.N, ea.K, ea.out_dt, 0, 0, &pl)) return st;
  const int grid_cap = g_gemm_sm_limit;
  const int kb = rung == APA_RUNG_FP8 ? 1 : rung == APA_RUNG_FP16 ? 2 : 4;
  TailPlan tp{0, 0, 0, 0, 0};
  if (pl.tile == kTilePair) {
    int cap = 0;
#define APA_CAP_CASE(KIND)                                                                                  \
  switch (epi) {                                                                                             \
    case EPI_FWD: cap = cap_of<KIND, EPI_FWD>(pl.ew); break;                                           \
    case EPI_DGRAD: cap = cap_of<KIND, EPI_DGRAD>(pl.ew); break;                                       \
    case EPI_RAW: cap = cap_of<KIND, EPI_RAW>(pl.ew); break;                                           \
    default: cap = cap_of<KIND, EPI_WGRAD>(pl.ew);                                                     \
  }
    switch (rung) {
      case APA_RUNG_FP8: APA_CAP_CASE(KIND_E4M3) break;
      case APA_RUNG_FP16: APA_CAP_CASE(KIND_F16) break;
      default: APA_CAP_CASE(KIND_TF32)
    }
#undef APA_CAP_CASE
    if (cap < 1) return APA_OK;
    const int slots = std::max(1, std::min(grid_cap > 0 ? std::max(1, grid_cap / 2) : cap, cap));
    tp = pl.ew == 8 ? tail_plan_for<256, true, 8>(ea, kb, slots) : tail_plan_for<256, true, 4>(ea, kb, slots);
  } else {
    const int slots = std::max(1, grid_cap > 0 ? grid_cap : num_sms());
    if (pl.tile == kTile256)
      tp = pl.ew == 8 ? tail_plan_for<256, false, 8>(ea, kb, slots) : tail_plan_for<256, false, 4>(ea, kb, slots);
    else
      tp = pl.ew == 8 ? tail_plan_for<128, false, 8>(ea, kb, slots) : tail_plan_for<128, false, 4>(ea, kb, slots);
  }
  *bytes_out = tp.splits > 1 ? tp.bytes : 0;
  return APA_OK;
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
  ea.out = nullptr; ea.ldo = 0; ea.out_dt = APA_DT_F32; ea.vec_out = 0; ea.tma_out = 0; ea.coalesced_out = 0;
  ea.bias = nullptr; ea.bias_vec = 0; ea.amax = nullptr; ea.flag = nullptr;
  ea.counters = nullptr; ea.ratio_max = nullptr; ea.vmin = 0.0f; ea.accumulate = 0; ea.finalize = 1; ea.telem = 0;
  ea.splits = 1; ea.kb_per_split = 0; ea.split_rows = 0;
  ea.sk_ws = nullptr; ea.sk_tickets = nullptr; ea.sk_ws_bytes = 0;
  ea.sk_first = 0; ea.sk_splits = 0; ea.sk_kb_per_split = 0;
  ea.dp = apa::dpr::RegionArgs{};
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
  const int bias_es = rung == APA_RUNG_FP8 ? 1 : rung == APA_RUNG_FP16 ? 2 : 4;
  ea.bias_vec = (reinterpret_cast<uintptr_t>(bias_q) % (uintptr_t)(4 * bias_es)) == 0 ? 1 : 0;
  ea.telem = (amax || flag) ? 1 : 0;
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
  ea.telem = (bc_amax || bc_flag) ? 1 : 0;
  return apa::gemm_dispatch(rung, apa::gemm::EPI_DGRAD, dyq, lddy, wqt, ldwt, ea, 0, 0,
                            static_cast<cudaStream_t>(stream));
}

namespace {

// The weight-gradient GEMM with its fused epilogue; `ws` (nullable, 16-byte
// aligned) lets the last partial wave of tiles be split along K (stream-K).
int wgrad_gemm(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt, float* dw, int64_t lddw,
               int64_t M, int64_t N, int64_t K, int accumulate, unsigned long long* counters, float* ratio_max,
               void* ws, int64_t ws_bytes, cudaStream_t s, const apa::dpr::RegionArgs* dp = nullptr) {
  EpiArgs ea = blank(N, K, M);
  if (dp != nullptr) ea.dp = *dp;
  ea.out = dw; ea.ldo = lddw; ea.out_dt = APA_DT_F32; ea.vec_out = out_vec(dw, lddw, 4);
  ea.accumulate = accumulate; ea.counters = counters; ea.ratio_max = ratio_max;
  ea.telem = counters ? 1 : 0;
  ea.vmin = rung == APA_RUNG_FP8 ? 0.015625f : rung == APA_RUNG_FP16 ? 6.1035e-5f : 0.0f;
  if (ws != nullptr && ws_bytes > 0 && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0) {
    ea.sk_ws = static_cast<float*>(ws);
    ea.sk_ws_bytes = ws_bytes;
  }
  return apa::gemm_dispatch(rung, apa::gemm::EPI_WGRAD, dyqt, lddyt, xqt, ldxt, ea, 0, 0, s);
}

}  // namespace

extern "C" int apa_linear_wgrad(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt, float* dw,
                                int64_t lddw, int64_t M, int64_t N, int64_t K, int accumulate,
                                unsigned long long* counters, float* ratio_max, void* stream) {
  // dw[N, K] = dyq[M, N]^T . xq[M, K]; operands are the transposed copies
  // dyqt[N, M] and xqt[K, M]; the GEMM reduces over M.
  if (int st = check_dims(N, K, M)) return st;
  if (!dyqt || !xqt || !dw || lddw < K || lddyt < M || ldxt < M) return APA_ERR_INVALID;
  if (rung != APA_RUNG_TF32 && !counters) return APA_ERR_INVALID;
  return wgrad_gemm(rung, dyqt, lddyt, xqt, ldxt, dw, lddw, M, N, K, accumulate, counters, ratio_max, nullptr, 0,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int apa_linear_wgrad_block(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt,
                                      float* dw, int64_t lddw, int64_t M, int64_t rows, int64_t K, int accumulate,
                                      unsigned long long* counters, float* ratio_max, int last, void* stream) {
  // rows [r0, r0 + rows) of dw[N, K]: dyqt and dw point at row r0 of dyq^T and dw
  if (int st = check_dims(rows, K, M)) return st;
  if (!dyqt || !xqt || !dw || lddw < K || lddyt < M || ldxt < M) return APA_ERR_INVALID;
  if (rung != APA_RUNG_TF32 && !counters) return APA_ERR_INVALID;
  EpiArgs ea = blank(rows, K, M);
  ea.out = dw; ea.ldo = lddw; ea.out_dt = APA_DT_F32; ea.vec_out = out_vec(dw, lddw, 4);
  ea.accumulate = accumulate; ea.counters = counters; ea.ratio_max = ratio_max;
  ea.finalize = last ? 1 : 0;
  ea.telem = counters ? 1 : 0;
  ea.vmin = rung == APA_RUNG_FP8 ? 0.015625f : rung == APA_RUNG_FP16 ? 6.1035e-5f : 0.0f;
  return apa::gemm_dispatch(rung, apa::gemm::EPI_WGRAD, dyqt, lddyt, xqt, ldxt, ea, 0, 0,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int apa_gemm_plan(int rung, int epilogue, int64_t M, int64_t N, int64_t K, int out_dtype, int tile,
                             int grid_cap, int* tile_out, int* epi_warps_out) {
  if (!tile_out || !epi_warps_out) return APA_ERR_INVALID;
  if (int st = check_dims(M, N, K)) return st;
  apa::GemmPlan pl;
  if (int st = apa::resolve_plan(rung, epilogue, M, N, K, out_dtype, tile, grid_cap, &pl)) return st;
  *tile_out = pl.tile;
  *epi_warps_out = pl.ew;
  return APA_OK;
}

extern "C" int apa_set_gemm_sm_limit(int limit) {
  if (limit < 0) return APA_ERR_INVALID;
  apa::g_gemm_sm_limit = limit;
  return APA_OK;
}

extern "C" int apa_set_pdl(int enabled) {
  if (enabled != 0 && enabled != 1) return APA_ERR_INVALID;
  apa::g_pdl = enabled;
  return APA_OK;
}

extern "C" int apa_gemm_tn(int rung, int epilogue, const void* A, int64_t lda, const void* B, int64_t ldb, void* out,
                           int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K, int tile, int grid_cap,
                           void* stream) {
  // Plain D = A . B^T with the epilogue of the given op and no telemetry
  // side effects; used to time the bare GEMM against the fused versions.
  if (int st = check_dims(M, N, K)) return st;
  if (!A || !B || !out) return APA_ERR_INVALID;
  EpiArgs ea = blank(M, N, K);
  ea.out = out; ea.ldo = ldo; ea.out_dt = out_dtype;
  ea.vec_out = out_vec(out, ldo, out_dtype == APA_DT_F32 ? 4 : 2);
  return apa::gemm_dispatch(rung, epilogue, A, lda, B, ldb, ea, tile, grid_cap, static_cast<cudaStream_t>(stream));
}

namespace apa {

// Split-K for a weight gradient dw[Mo, No] reduced over Kt tokens: used when
// the tiles of the ordinary plan would keep fewer than half of the SMs busy
// and the reduction is long; each split then covers at least 16 K slabs.
struct SplitPlan {
  int tile, ew, splits, kb_per_split;
  int64_t ld_ws;       // row pitch of a slice (16-byte rows)
  int64_t rows_pad;    // rows of a slice: the epilogue stores 32-row boxes, so a
                       // slice is padded to a multiple of 32 and no box of one
                       // split reaches into the next split's slice
};

SplitPlan plan_wgrad_split(int rung, int64_t Mo, int64_t No, int64_t Kt) {
  using namespace gemm;
  SplitPlan sp{0, 0, 1, 0, 0, 0};
  const int es = rung == APA_RUNG_FP8 ? 1 : rung == APA_RUNG_FP16 ? 2 : 4;
  const int slots = g_gemm_sm_limit > 0 ? g_gemm_sm_limit : num_sms();
  GemmPlan pl = plan_gemm(Mo, No, Kt, es, 4, slots, false, 0, gemm::EPI_WGRAD);
  auto cdiv = [](int64_t a, int64_t b) { return (a + b - 1) / b; };
  const int64_t tiles = cdiv(Mo, 128) * cdiv(No, pl.tile == kTile128 ? 128 : 256);
  const int64_t kb_count = cdiv(Kt * es, kSlab);
  if (tiles * 2 > slots) return sp;
  int64_t S = std::min<int64_t>(std::min<int64_t>(slots / tiles, 8), kb_count / 16);
  if (S < 2) return sp;
  const int64_t per = cdiv(kb_count, S);
  S = cdiv(kb_count, per);
  if (S < 2) return sp;
  sp.tile = pl.tile;
  sp.ew = 8;   // a single wave: the epilogue is exposed
  sp.splits = (int)S;
  sp.kb_per_split = (int)per;
  sp.ld_ws = (No + 3) / 4 * 4;
  sp.rows_pad = (Mo + 31) / 32 * 32;
  return sp;
}

}  // namespace apa

extern "C" int apa_wgrad_workspace_bytes(int rung, int64_t M, int64_t N, int64_t K, int64_t* bytes_out) {
  if (!bytes_out) return APA_ERR_INVALID;
  if (int st = check_dims(N, K, M)) return st;
  if (rung != APA_RUNG_FP8 && rung != APA_RUNG_FP16 && rung != APA_RUNG_TF32) return APA_ERR_INVALID;
  const apa::SplitPlan sp = apa::plan_wgrad_split(rung, N, K, M);
  if (sp.splits > 1) {
    *bytes_out = (int64_t)sp.splits * sp.rows_pad * sp.ld_ws * 4;
    return APA_OK;
  }
  // otherwise the stream-K split of the last partial wave, if it has one
  EpiArgs ea = blank(N, K, M);
  ea.out_dt = APA_DT_F32;
  return apa::tail_workspace_bytes(rung, apa::gemm::EPI_WGRAD, ea, bytes_out);
}

namespace apa {
// dp_nvls.cu: publish every region of a gradient (defer_owned: and hand this
// rank's own to the deferred pass)
int dp_region_signal(const dpr::RegionArgs& a, int defer_owned, cudaStream_t s);
}  // namespace apa

namespace {

// Whether this weight gradient is computed split along the tokens (two
// kernels: fp32 partials into the workspace, then their ordered sum with the
// weight-gradient epilogue) and the workspace is enough for it.
bool wgrad_is_split(const apa::SplitPlan& sp, int64_t N, int64_t K, const void* workspace, int64_t workspace_bytes) {
  const int64_t need = sp.splits > 1 ? (int64_t)sp.splits * sp.rows_pad * sp.ld_ws * 4 : 0;
  // the reduction kernel takes at most 8 splits and 32-bit element indices
  // (the plan only splits outputs of a few tiles, so neither limit is reached)
  return !(need == 0 || !workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u) ||
           N * K >= (1ll << 31) || sp.splits > 8);
}

int wgrad_split(const apa::SplitPlan& sp, int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt,
                float* dw, int64_t lddw, int64_t M, int64_t N, int64_t K, int accumulate,
                unsigned long long* counters, float* ratio_max, void* workspace, cudaStream_t s) {
  // phase 1: raw fp32 partial sums, one slice per split
  EpiArgs ea = blank(N, K, M);
  ea.out = workspace; ea.ldo = sp.ld_ws; ea.out_dt = APA_DT_F32; ea.vec_out = 1;
  ea.splits = sp.splits; ea.kb_per_split = sp.kb_per_split; ea.split_rows = (int)sp.rows_pad;
  const int tile = sp.tile | (sp.ew == 8 ? apa::gemm::kEpiFlag8 : apa::gemm::kEpiFlag4);
  if (int st = apa::gemm_dispatch(rung, apa::gemm::EPI_RAW, dyqt, lddyt, xqt, ldxt, ea, tile, 0, s)) return st;
  // phase 2: ordered sum + the weight-gradient epilogue
  const float vmin = rung == APA_RUNG_FP8 ? 0.015625f : rung == APA_RUNG_FP16 ? 6.1035e-5f : 0.0f;
  const bool vec = (K % 4) == 0 && (lddw % 4) == 0 && (reinterpret_cast<uintptr_t>(dw) & 15u) == 0;
  const int64_t total = vec ? N * K / 4 : N * K;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)apa::num_sms() * 4));
  const float* ws = static_cast<const float*>(workspace);
  const int64_t slice = sp.rows_pad * sp.ld_ws;
  using namespace apa::gemm;
#define APA_WGRAD_REDUCE(KIND_)                                                                             \
  apa::launch_kernel(vec ? wgrad_reduce_kernel<KIND_, true> : wgrad_reduce_kernel<KIND_, false>, dim3(grid),\
                     dim3(256), 0, s, 1, ws, sp.splits, slice, sp.ld_ws, (int)N, (int)K, dw, lddw, accumulate,   \
                     vmin, counters, ratio_max);
  switch (rung) {
    case APA_RUNG_FP8: APA_WGRAD_REDUCE(KIND_E4M3) break;
    case APA_RUNG_FP16: APA_WGRAD_REDUCE(KIND_F16) break;
    default: APA_WGRAD_REDUCE(KIND_TF32)
  }
#undef APA_WGRAD_REDUCE
  return cudaGetLastError() == cudaSuccess ? APA_OK : APA_ERR_CUDA;
}

}  // namespace

extern "C" int apa_linear_wgrad_ws(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt, float* dw,
                                   int64_t lddw, int64_t M, int64_t N, int64_t K, int accumulate,
                                   unsigned long long* counters, float* ratio_max, void* workspace,
                                   int64_t workspace_bytes, void* stream) {
  if (int st = check_dims(N, K, M)) return st;
  if (!dyqt || !xqt || !dw || lddw < K || lddyt < M || ldxt < M) return APA_ERR_INVALID;
  if (rung != APA_RUNG_TF32 && !counters) return APA_ERR_INVALID;
  const apa::SplitPlan sp = apa::plan_wgrad_split(rung, N, K, M);
  if (!wgrad_is_split(sp, N, K, workspace, workspace_bytes))
    return wgrad_gemm(rung, dyqt, lddyt, xqt, ldxt, dw, lddw, M, N, K, accumulate, counters, ratio_max, workspace,
                      workspace_bytes, static_cast<cudaStream_t>(stream));
  return wgrad_split(sp, rung, dyqt, lddyt, xqt, ldxt, dw, lddw, M, N, K, accumulate, counters, ratio_max, workspace,
                     static_cast<cudaStream_t>(stream));
}

extern "C" int apa_linear_wgrad_dp(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt,
                                   float* dw, int64_t lddw, int64_t M, int64_t N, int64_t K,
                                   unsigned long long* counters, float* ratio_max, void* workspace,
                                   int64_t workspace_bytes, float* dw_mc, const unsigned int* ready_local,
                                   unsigned int* ready_mc, unsigned int* done_mc, const unsigned int* epoch_local,
                                   unsigned int* deferred_local, int world, int rank, void* stream) {
  if (int st = check_dims(N, K, M)) return st;
  if (!dyqt || !xqt || !dw || lddw < K || lddyt < M || ldxt < M) return APA_ERR_INVALID;
  if (rung != APA_RUNG_TF32 && !counters) return APA_ERR_INVALID;
  apa::dpr::RegionArgs dp;
  if (int st = apa::dpr::make_region_args(&dp, dw_mc, lddw, N, K, ready_local, ready_mc, done_mc, epoch_local,
                                          deferred_local, world, rank))
    return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const apa::SplitPlan sp = apa::plan_wgrad_split(rung, N, K, M);
  if (!wgrad_is_split(sp, N, K, workspace, workspace_bytes))
    return wgrad_gemm(rung, dyqt, lddyt, xqt, ldxt, dw, lddw, M, N, K, 0, counters, ratio_max, workspace,
                      workspace_bytes, s, &dp);
  // split along the tokens: the gradient is complete after the second
  // kernel, then the standalone form of the same regions
  if (int st = wgrad_split(sp, rung, dyqt, lddyt, xqt, ldxt, dw, lddw, M, N, K, 0, counters, ratio_max, workspace, s))
    return st;
  // kernel, then its regions published with this rank's own marked deferred
  // (the caller's side-stream pass averages them; nothing waits here)
  return apa::dp_region_signal(dp, 1, s);
}
