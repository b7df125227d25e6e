/*
 * C ABI of libapa_kernels.so: the B200 (sm_100a) kernels behind the APA
 * per-layer precision path. Plain pointers, sizes and a cudaStream_t passed
 * as void*; no framework types. Every entry point returns an APA_* status
 * (0 on success) and never exits or traps. Device pointers are caller-owned
 * (the Python layer allocates them with torch's caching allocator); the
 * kernels allocate nothing.
 *
 * Shapes are row-major with an explicit leading dimension (elements).
 * Reference = Adaptive Precision Ascension, apa/ (file:line cited per entry).
 */
#ifndef APA_KERNELS_H
#define APA_KERNELS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define APA_OK 0
#define APA_ERR_INVALID 1     /* null pointer, negative/zero size, leading dimension too small */
#define APA_ERR_ALIGN 2       /* operand not 16-byte aligned where the TMA path needs it */
#define APA_ERR_UNSUPPORTED 3 /* dtype / rung combination not provided */
#define APA_ERR_CUDA 4        /* launch failure or missing driver entry point */
#define APA_ERR_NOALLOC_LIMIT 5 /* problem larger than apa_bias_grad_noalloc's fixed scratch */

/* element types */
#define APA_DT_F32 0
#define APA_DT_F16 1
#define APA_DT_BF16 2
#define APA_DT_E4M3 3
#define APA_DT_TF32 4 /* apa_cast destination only: fp32 storage rounded to the TF32
                         grid (round half to even), the operand form of the TF32 rung */

/* ladder rungs, apa/config.py:5-7 (LEVEL_FP8, LEVEL_FP16, LEVEL_TF32) */
#define APA_RUNG_FP8 0
#define APA_RUNG_FP16 1
#define APA_RUNG_TF32 2

/* GEMM epilogues for apa_gemm_tn */
#define APA_EPI_FWD 0
#define APA_EPI_DGRAD 1
#define APA_EPI_WGRAD 2
#define APA_EPI_RAW 3   /* plain fp32 accumulator (split-K partials, bare timing) */

/* Library ABI version (bumped on any signature change). */
int apa_abi_version(void);

/* Human-readable text for a status code. */
const char* apa_status_string(int status);

/* Read (and optionally clear) the device status word that bounded waits set
 * when they give up. 0 means no kernel has timed out. Synchronous. */
int apa_get_device_status(unsigned int* out, int clear);

/*
 * Cast a [rows, cols] matrix to dst_dtype with fused telemetry.
 * Replaces: APABoundaryCast.forward x.to(working_dtype) (apa/layers.py:17-21),
 * APALinear.refresh_working_copy weight_master.to(dtype) (layers.py:368-372),
 * the E4M3 cast of grad_output in backward (layers.py:225, :243), and the
 * track_telemetry_on_tensor pass on each of those tensors (telemetry.py:7-21,
 * called at layers.py:142-143, :211).
 *   dst / dst_t        nullable: row-major copy and transposed copy [cols, rows]
 *   amax, flag         nullable: running NaN-propagating max of |value| and
 *                      max(flag, 1) on any NaN/Inf, over the cast values, or
 *                      over the source values when telem_on_source != 0
 *   merge_amax         nullable: a pending amax (e.g. the weight's, taken when
 *                      the working copy was made) merged into amax/flag
 *   colsum_partial     nullable: [ceil(rows/64), cols] fp32 partial column
 *                      sums of the cast values (bias gradient, layers.py:241)
 * src_dtype: F32, F16 or BF16; dst_dtype: E4M3, F16, F32, TF32 (BF16 also
 * accepted). With TF32 the stored values are rounded to the TF32 grid while
 * telemetry and column sums use the unrounded fp32 values (the reference's
 * TF32 rung computes in true fp32).
 */
int apa_cast(const void* src, int src_dtype, int64_t rows, int64_t cols, int64_t ld_src,
             void* dst, int dst_dtype, int64_t ld_dst, void* dst_t, int64_t ld_dst_t,
             float* amax, int32_t* flag, int telem_on_source, const float* merge_amax,
             float* colsum_partial, void* stream);

/* amax / nonfinite telemetry of a flat array of n elements of dtype.
 * Replaces: track_telemetry_on_tensor (apa/telemetry.py:7-21) where no fused
 * kernel produced the tensor (APALinear.track_telemetry, layers.py:374-389;
 * the non-APA backward hooks, manager.py:79-84). */
int apa_amax(const void* src, int dtype, int64_t n, float* amax, int32_t* flag, void* stream);

/* Underflow ratio of a flat array: #(0 < |g| < vmin) / #(|g| > 0) in fp32,
 * 0 when nothing is nonzero; stored in *ratio_out, or folded into it as a
 * running max when running_max != 0. counters: 3 zeroed u64 scratch words,
 * zero again on return.
 * Replaces: compute_underflow_ratio (apa/telemetry.py:23-39) and
 * APALinear.update_underflow_metric (apa/layers.py:404-407) when called on a
 * tensor outside the fused weight-gradient GEMM. */
int apa_underflow_ratio(const void* src, int dtype, int64_t n, float vmin, unsigned long long* counters,
                        float* ratio_out, int running_max, void* stream);

/* Fold a stored amax into a telemetry pair (amax max, flag if non-finite). */
int apa_merge_telemetry(float* amax, int32_t* flag, const float* src_amax, void* stream);

/* Bias gradient from apa_cast's colsum_partial: sum the nparts rows of
 * partials per column, round to work_dtype (the engine's cast to bias_work's
 * dtype) and write the fp32 value to out (bias_master.grad), or add it when
 * accumulate != 0.
 * Replaces: grad_bias in APALinearFunction.backward (layers.py:239-241,
 * :265-266, :274-275, :290-291) and its copy in _sync_grads_to_master
 * (manager.py:200-204). */
int apa_colsum_finalize(const float* partial, int64_t nparts, int64_t cols, int work_dtype,
                        float* out, int accumulate, void* stream);

/* Set n int32 device words (given by a device array of pointers) to zero.
 * Replaces: the per-step flag resets in APAManager.pre_step (manager.py:161-168). */
int apa_zero_list(int32_t* const* ptrs, int n, void* stream);

/*
 * Forward GEMM: y[M,N] = xq[M,K] . wq[N,K]^T + bias, fused amax/NaN telemetry
 * of y into amax/flag.
 * Replaces: APALinearFunction.forward's per-rung GEMM (layers.py:158-182,
 * _call_scaled_mm layers.py:23-60) and track_telemetry_on_tensor(result)
 * (layers.py:186).
 * rung FP8: xq, wq E4M3, bias E4M3 (nullable), y fp32.
 * rung FP16: xq, wq, bias fp16, y fp16.  rung TF32: all fp32.
 * xq and wq rows must be 16-byte aligned (ld * element size % 16 == 0).
 */
int apa_linear_fwd(int rung, const void* xq, int64_t ldx, const void* wq, int64_t ldw,
                   const void* bias_q, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                   float* amax, int32_t* flag, void* stream);

/*
 * Input-gradient GEMM: dx[M,K] = cast(cast(dyq[M,N] . wq[N,K], working dtype), dx_dtype).
 * wqt is the transposed working weight [K, N]. bc_amax / bc_flag (nullable)
 * receive the telemetry of the working-dtype gradient.
 * Replaces: grad_input in APALinearFunction.backward (layers.py:233-234,
 * :247-255, :268-269, :277-278), the autograd engine's cast of it to x_cast's
 * dtype, ToCopyBackward to x's dtype, and the boundary_cast backward hook's
 * track_telemetry_on_tensor (manager.py:79-84).
 */
int apa_linear_dgrad(int rung, const void* dyq, int64_t lddy, const void* wqt, int64_t ldwt,
                     void* dx, int dx_dtype, int64_t lddx, int64_t M, int64_t N, int64_t K,
                     float* bc_amax, int32_t* bc_flag, void* stream);

/*
 * Weight-gradient GEMM: dw[N,K] = f32(cast(dyq[M,N]^T . xq[M,K], working dtype))
 * from the transposed operands dyqt[N,M] and xqt[K,M]; accumulate != 0 adds
 * into dw. Counts the nonzero and below-threshold elements of the unrounded
 * (FP16: fp16-rounded) gradient in counters[0..1] (counters[2] is a CTA
 * ticket; all three must be zero on entry and are zero again on return), and
 * the last CTA folds counters[1]/counters[0] into *ratio_max as a running max.
 * Thresholds: 2^-6 (FP8), 6.1035e-5 (FP16), 0 (TF32: no counting).
 * Replaces: grad_weight in APALinearFunction.backward (layers.py:235-238,
 * :256-264, :270-273, :279-282), compute_underflow_ratio (telemetry.py:23-39)
 * with its per-layer .item() sync, update_underflow_metric (layers.py:404-407)
 * and the weight half of _sync_grads_to_master (manager.py:191-199).
 */
int apa_linear_wgrad(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt,
                     float* dw, int64_t lddw, int64_t M, int64_t N, int64_t K, int accumulate,
                     unsigned long long* counters, float* ratio_max, void* stream);

/*
 * apa_linear_wgrad for a block of output rows: dyqt and dw point at row r0 of
 * dyq^T [N, M] and dw [N, K], and rows output rows are computed. The counts
 * accumulate in counters across blocks; only the call with last != 0 folds
 * counters[1]/counters[0] into *ratio_max and zeroes them, so a gradient made
 * in row blocks yields the same values and the same ratio as one call. Lets a
 * data-parallel backward start the all-reduce of finished rows while the next
 * rows are computed. Same reference interfaces as apa_linear_wgrad.
 */
int apa_linear_wgrad_block(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt,
                           float* dw, int64_t lddw, int64_t M, int64_t rows, int64_t K, int accumulate,
                           unsigned long long* counters, float* ratio_max, int last, void* stream);

/*
 * Scratch bytes apa_linear_wgrad_ws uses for this shape (same M, N, K as
 * apa_linear_wgrad), 0 when the weight gradient is not split (neither along
 * the tokens for a small gradient, nor in its last partial wave of tiles).
 */
int apa_wgrad_workspace_bytes(int rung, int64_t M, int64_t N, int64_t K, int64_t* bytes_out);

/*
 * apa_linear_wgrad with a caller-owned scratch buffer (16-byte aligned,
 * apa_wgrad_workspace_bytes long): when the weight gradient's tiles would
 * leave most SMs idle (small N x K, many tokens), the reduction over tokens is
 * split into up to 8 parts computed in parallel as fp32 partial sums, then
 * summed in split order by a second kernel that applies the same epilogue
 * (underflow counts, rounding to the working dtype, overwrite or accumulate,
 * ratio fold). Otherwise, when the persistent schedule's last wave of tiles is
 * at most half full (e.g. 4096 x 4096 over 8192 tokens: 256 tiles on 74 CTA
 * pairs), each tile of that wave is split in two along the tokens (stream-K):
 * both halves run side by side, store their fp32 partial sums in the scratch
 * buffer, and the half that finishes second adds the two (the same bits
 * whichever finishes first) and applies the epilogue. The entry point clears
 * the scratch words it needs itself. Without enough scratch it behaves exactly
 * like apa_linear_wgrad. Same reference interfaces as apa_linear_wgrad.
 */
int apa_linear_wgrad_ws(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt,
                        float* dw, int64_t lddw, int64_t M, int64_t N, int64_t K, int accumulate,
                        unsigned long long* counters, float* ratio_max, void* workspace,
                        int64_t workspace_bytes, void* stream);

/*
 * Cap the number of CTAs (SMs) the persistent GEMMs use; 0 restores one CTA
 * per SM. Process-wide. The data-parallel path sets it while a gradient
 * all-reduce runs alongside a GEMM so the collective's kernel finds free SMs.
 * No counterpart in the reference (it has no gradient collective).
 */
int apa_set_gemm_sm_limit(int limit);

/*
 * Launch mode of every kernel of the library except the data-parallel NVLS
 * ones: 1 (the default) = programmatic dependent launch, so a kernel's launch
 * and prologue overlap the end of the kernel before it in the stream or CUDA
 * graph (each kernel waits for that kernel's completion before it touches
 * global memory); 0 = plain stream order. Affects launches made after the
 * call. No counterpart in the reference.
 */
int apa_set_pdl(int enabled);

/*
 * The same tcgen05 GEMM with a chosen epilogue and no telemetry side effects,
 * a chosen tile shape (APA_TILE_*; APA_TILE_AUTO picks one) and grid cap in
 * CTAs (0 = one CTA per SM). Used to time the bare GEMM against the fused
 * entry points and to test every tile shape. APA_ERR_UNSUPPORTED when the
 * CTA-pair shape cannot be launched on this device.
 */
#define APA_TILE_AUTO 0
#define APA_TILE_128x128 128      /* one CTA per tile */
#define APA_TILE_128x256 256      /* one CTA per tile */
#define APA_TILE_PAIR_256x256 512 /* a cluster of two CTAs, tcgen05 cta_group::2 */
/* OR-ed into the tile code: the number of epilogue warps (default: chosen
 * with the tile, 8 when the epilogue cannot hide behind the MMAs) */
#define APA_TILE_EPI_WARPS_4 1
#define APA_TILE_EPI_WARPS_8 2
int apa_gemm_tn(int rung, int epilogue, const void* A, int64_t lda, const void* B, int64_t ldb,
                void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                int tile, int grid_cap, void* stream);

/*
 * The launch configuration a GEMM of this shape would use (apa_linear_* pass
 * APA_TILE_AUTO and grid cap 0; M, N, K as in apa_gemm_tn, i.e. for dgrad
 * M = tokens, N = in features, K = out features and for wgrad M = out
 * features, N = in features, K = tokens): *tile_out = 128, 256 or 512
 * (APA_TILE_*), *epi_warps_out = 4 or 8. Launches nothing. No counterpart in
 * the reference.
 */
int apa_gemm_plan(int rung, int epilogue, int64_t M, int64_t N, int64_t K, int out_dtype, int tile,
                  int grid_cap, int* tile_out, int* epi_warps_out);

/*
 * AdamW on an fp32 master weight [rows, cols] (row pitch ld, shared by p, g,
 * m, v) fused with the next step's working copy: p, m, v updated in place in
 * torch.optim.AdamW's order of operations (decoupled decay, bias-corrected
 * step `step` >= 1) and, in the same pass, the updated p cast to work_dtype
 * (E4M3, F16 or TF32) into wq and/or its transpose wq_t, with max |cast
 * value| written to *w_amax (which is reset first). Every row pitch and base
 * address must be 16-byte aligned (TMA tiles in and out); APA_ERR_UNSUPPORTED
 * otherwise. Replaces the optimizer
 * step plus the weight half of the working-copy refresh in pre_step
 * (manager.py:145-172, layers.py:368-372).
 */
int apa_adamw_cast(float* p, const float* g, float* m, float* v, int64_t rows, int64_t cols, int64_t ld,
                   float lr, float beta1, float beta2, float eps, float weight_decay, int64_t step,
                   void* wq, int work_dtype, int64_t ld_q, void* wq_t, int64_t ld_qt, float* w_amax,
                   void* stream);

/*
 * Forensic statistics of a flat tensor of n elements (n < 2^32) into a
 * 5-word device record (zeroed here): [0] (max |x| fp32 bits << 32) | ~index
 * of its first occurrence (NaN ranks largest), [1] sum and [2] sum of squares
 * as fp64, [3] n, [4] 1 if any element is NaN or infinite. No host
 * synchronisation. Replaces the per-tensor .item() reads of forensic mode
 * (layers.py:63-106: amax, mean, std, argmax per tensor role).
 */
int apa_tensor_stats(const void* src, int dtype, int64_t n, unsigned long long* record, void* stream);

/*
 * Bias gradient without any device allocation: db[c] = f32(cast(sum_r
 * f32(cast(dy[r, c], work)), work)) (or += when accumulate != 0), the same
 * result as apa_cast with colsum_partial followed by apa_colsum_finalize.
 * No counterpart in the reference: this entry point exists for callers that
 * cannot allocate device memory when they call (a host framework that owns
 * all device memory, code running amid another runtime's queued stream work
 * where cudaMalloc/cudaFree would synchronise the device, foreign-language
 * bindings holding only borrowed device pointers). Its partial sums live in a
 * fixed 16 MiB array inside the library, kept by every GPU that loads it:
 * ceil(rows / 64) * cols must not exceed 4 Mi (else APA_ERR_NOALLOC_LIMIT).
 * All calls share that array, so calls that overlap on the GPU race; the first
 * call on a device looks up the array's device address and should come before
 * any stream capture (so should the first call after the device's context was
 * replaced, e.g. by cudaDeviceReset: the address is looked up again then). It
 * calls no cudaMalloc/cudaFree.
 * dy_dtype: F32, F16 or BF16; work_dtype: E4M3, F16 or F32.
 */
int apa_bias_grad_noalloc(const void* dy, int dy_dtype, int64_t rows, int64_t cols, int64_t ld,
                          int work_dtype, float* db, int accumulate, void* stream);

/*
 * Ladder evaluation on device, one launch per step.
 * Replaces: APAManager._check_hard_overflow (manager.py:178-189),
 * _do_full_evaluation (manager.py:206-261) and _escalate_module's level/EMA
 * update (manager.py:267-293); the host then needs one small read of `out`
 * instead of 3 .item() syncs per module.
 *
 * Inputs per APA module i < L (device arrays): amax_ptr[i], ratio_ptr[i],
 * flag_ptr[i] point at the module's gpu_amax / gpu_underflow_ratio /
 * gpu_has_nonfinite; level[i] (int32) and ema[i] (double) are the ladder state,
 * updated in place. Per non-APA leaf j < O: oamax_ptr[j], oflag_ptr[j].
 * `global` (nullable, int32[1 + 3L + 2O]): when given, the telemetry is read
 * from this already-reduced vector (see apa_ladder_pack) instead of the
 * pointers, so every data-parallel rank decides identically.
 * `out` (device memory; int32[4 + 2L + O], padded to 8 bytes, then
 * double[2L + O]) receives the decision record the host uses for logging;
 * when `out_host` (pinned host memory) is given the record is also copied there
 * on the same stream, so the host needs one stream synchronisation.
 */
/*
 * Data-parallel averaging of an fp32 weight gradient [rows, cols] (row pitch
 * ld; cols and ld multiples of 4, 16-byte aligned) through NVLink SHARP. The
 * gradient of every rank lives at the same offset of a symmetric allocation
 * bound to an NVLink multicast object; grad_mc and *_mc are multicast
 * addresses in it, *_local this rank's own words (u32, zero at start): one
 * ready counter and one deferred word per region (apa_dp_regions: regions of
 * 32 rows x 64 columns, region g averaged by rank g % world), one done
 * counter and one epoch word per gradient. Per gradient and step, on every
 * rank:
 *   either apa_linear_wgrad_dp (the GEMM runs the protocol in its epilogue)
 *     and, on a side stream after it, apa_dp_region_reduce with
 *     only_deferred = 1 (the regions a split gradient left to it),
 *   or, after the gradient is written some other way, apa_dp_region_signal on
 *     the stream that wrote it and apa_dp_region_reduce (only_deferred = 0)
 *     after it;
 *   then apa_dp_region_wait: waits until every region is averaged (done
 *     reaches regions x (epoch + 1)), then advances the epoch; work queued
 *     after it sees the mean over ranks in every rank's gradient.
 * Every rank must run the same gradients in the same order (each waits in
 * its GEMM's epilogue for the others' regions). Waits are bounded (2 s); on
 * expiry the library status word is set (see apa_get_device_status; the
 * ladder's decision record reports it), the waiter still signals, later
 * waits give up at once, and the kernels return. Ranks may mix the two forms.
 * No counterpart in the reference (it has no gradient collective; its only
 * collective is the flag all-reduce, manager.py:186-187).
 */
int apa_dp_regions(int64_t rows, int64_t cols, int64_t* regions_out);
int apa_dp_region_signal(float* grad_mc, int64_t ld, int64_t rows, int64_t cols, const unsigned int* ready_local,
                         unsigned int* ready_mc, unsigned int* done_mc, const unsigned int* epoch_local,
                         unsigned int* deferred_local, int world, int rank, void* stream);
int apa_dp_region_reduce(float* grad_mc, int64_t ld, int64_t rows, int64_t cols, const unsigned int* ready_local,
                         unsigned int* ready_mc, unsigned int* done_mc, const unsigned int* epoch_local,
                         unsigned int* deferred_local, int world, int rank, int only_deferred, int ctas,
                         void* stream);
int apa_dp_region_wait(const unsigned int* done_local, unsigned int* epoch_local, int64_t regions, void* stream);

/*
 * Weight gradient and its data-parallel average in one kernel: dw = this
 * rank's gradient exactly as apa_linear_wgrad_ws computes it (accumulate = 0;
 * counters and ratio_max of this rank's gradient), then every 32 x 64 region
 * of it, as soon as this rank's values are stored, published to the other
 * ranks, and the regions this rank owns averaged through the switch by the
 * same epilogue warps while the tensor cores compute later tiles. dw_mc is the multicast
 * address of dw; the counters as for apa_dp_region_*. Work that reads dw
 * queues after apa_dp_region_wait. Shapes whose weight gradient is split
 * along the tokens take the split kernels, then publish every region and
 * defer this rank's own, inside this call. Replaces the same step as
 * apa_linear_wgrad_ws followed by the gradient all-reduce.
 */
int apa_linear_wgrad_dp(int rung, const void* dyqt, int64_t lddyt, const void* xqt, int64_t ldxt, float* dw,
                        int64_t lddw, int64_t M, int64_t N, int64_t K, unsigned long long* counters,
                        float* ratio_max, void* workspace, int64_t workspace_bytes, float* dw_mc,
                        const unsigned int* ready_local, unsigned int* ready_mc, unsigned int* done_mc,
                        const unsigned int* epoch_local, unsigned int* deferred_local, int world, int rank,
                        void* stream);

int apa_ladder_pack(int L, const float* const* amax_ptr, const float* const* ratio_ptr,
                    const int32_t* const* flag_ptr, int O, const float* const* oamax_ptr,
                    const int32_t* const* oflag_ptr, int32_t* packed, void* stream);

int apa_ladder_eval(int L, float* const* amax_ptr, float* const* ratio_ptr, int32_t* const* flag_ptr,
                    int32_t* level, double* ema, int O, float* const* oamax_ptr, int32_t* const* oflag_ptr,
                    const int32_t* global, int64_t step_count, int64_t check_interval, double theta,
                    double alpha, void* out, void* out_host, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* APA_KERNELS_H */
