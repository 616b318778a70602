/*
 * smeai_q2k.h -- C-ABI of the sm_100a Q2_K x Q8_K mul_mat path.
 *
 * Replaces the ggml 0.9.8 Q2_K matrix-multiply path that the reference grafts
 * into llama.cpp (llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:82-136,
 * docs/architecture.md:41-46).  ggml's own sources are not part of the
 * reference tree; the ggml-shaped entry points below keep the signatures of
 * ggml's CPU type traits so a ggml build can bind them in place of its own.
 *
 * Two groups of entry points:
 *
 *  1. ggml-shaped (host pointers, ggml's block layouts, ggml's semantics).
 *     Each call stages its data to the GPU, runs the same kernels as the
 *     coarse entry points, and copies the result back.  They cannot report
 *     errors (ggml's signatures return void); on failure they leave the
 *     outputs zeroed and smeai_last_error() says why.  They are reentrant:
 *     each calling thread gets its own stream and staging buffers.
 *
 *  2. Coarse GPU entry points (device pointers, explicit stream, int status:
 *     0 = OK, negative = the sme_ai_status codes of sme_ai_ops.h, -5 = CUDA
 *     error).  Weights are repacked once into a device-resident tile layout
 *     (the analogue of ggml's CPU_REPACK extra buffer type) and referenced by
 *     an opaque handle.
 *
 * Block layouts (bytes):  block_q2_K = scales[16] qs[64] d(fp16) dmin(fp16)
 *                         = 84 per 256 weights;
 *                         block_q8_K = d(f32) qs[256](int8) bsums[16](int16)
 *                         = 292 per 256 activations.
 * Streams are passed as `void *` (a cudaStream_t; NULL = legacy default).
 */
#ifndef SMEAI_Q2K_H
#define SMEAI_Q2K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SMEAI_QK_K 256
#define SMEAI_BLOCK_Q2_K_BYTES 84
#define SMEAI_BLOCK_Q8_K_BYTES 292

/* ---------------- 1. ggml type-trait shaped entry points ----------------- */

/* Replaces ggml-cpu quantize_row_q8_K (generic C quantize_row_q8_K_ref):
 * k floats (k % 256 == 0) -> k/256 block_q8_K at y. */
void quantize_row_q8_K(const float *x, void *y, int64_t k);

/* Replaces ggml-quants.c quantize_row_q2_K_ref (Q2_K from_float). */
void quantize_row_q2_K(const float *x, void *y, int64_t k);

/* Replaces ggml-quants.c dequantize_row_q2_K (Q2_K to_float). */
void dequantize_row_q2_K(const void *x, float *y, int64_t k);

/* Replaces ggml-cpu ggml_vec_dot_q2_K_q8_K (type_traits_cpu[Q2_K].vec_dot):
 * *s = dot(row vx, row vy) over n values (n % 256 == 0).  nrc must be 1
 * (ggml never requests more for Q2_K); bs, bx, by are then unused. */
void ggml_vec_dot_q2_K_q8_K(int n, float *s, size_t bs, const void *vx, size_t bx, const void *vy, size_t by,
                            int nrc);

/* ---------------- 2. coarse GPU entry points ----------------------------- */

/* Is a compute-capability-10.x device present and usable?  1 / 0. */
int smeai_device_ready(void);

/* Text of the last error raised on the calling thread ("" if none). */
const char *smeai_last_error(void);

/* Limits of the kernels' bounded waits for kernels launched after this call:
 * local_ns for waits on this GPU's own work (default 2 s), peer_ns for waits
 * on rows other GPUs store (default 10 s); 0 keeps the default.  Production
 * code leaves the defaults; tests shorten a limit to make a wait run out
 * (a kernel captured in a CUDA graph keeps the limits of its capture). */
void smeai_set_wait_timeouts(uint64_t local_ns, uint64_t peer_ns);

/* Test hook: the library's next n device allocations fail as cudaMalloc does
 * when the device is out of memory (the entry points then return
 * SME_AI_ALLOC_FAILED / -2).  0 turns it off. */
void smeai_debug_fail_next_allocs(int n);

/* Reads and clears the current device's error word.  Kernels never trap or
 * spin forever: a wait that exceeds its time bound sets bit 0 (timeout) here
 * and the kernel returns early, leaving its outputs incomplete.  Returns 0,
 * or a negative status if the word cannot be read. */
int smeai_take_device_error(unsigned *code);

/* Repack n_rows x k of block_q2_K (row-major, host or device memory) into the
 * device tile layout; *w_dev_out receives an opaque handle.  The analogue of
 * ggml's CPU_REPACK buffer placement (q2_K_8x8_q8_K traits). */
int smeai_q2k_repack(const void *w_q2k, int64_t n_rows, int64_t k, void **w_dev_out);
void smeai_q2k_free(void *w_dev);
/* Device bytes held by a repacked weight. */
size_t smeai_q2k_weight_bytes(const void *w_dev);

/* Q8_K quantization of n_cols rows of k floats (device memory, row stride
 * ld_x floats) into n_cols * k/256 contiguous block_q8_K. */
int smeai_q8k_quantize(const float *x_dev, int64_t ld_x, int64_t n_cols, int64_t k, void *y_q8k_dev,
                       void *stream);
/* The same after an RMSNorm of each row: x / sqrt(mean(x^2) + eps)
 * (sme_ai_library/src/sme_ai_ops.c:1060-1092), fused into one kernel. */
int smeai_rms_q8k_quantize(const float *x_dev, int64_t ld_x, int64_t n_cols, int64_t k, float eps,
                           void *y_q8k_dev, void *stream);
/* The same with the RMSNorm weight of the reference's sme_ai_rmsnorm_f32
 * (sme_ai_ops.c:1084-1086): x * inv_rms, then times weight[j] (k floats on the
 * device; NULL = none), each product rounded once, then Q8_K. */
int smeai_rms_q8k_quantize_w(const float *x_dev, int64_t ld_x, int64_t n_cols, int64_t k, const float *weight_dev,
                             float eps, void *y_q8k_dev, void *stream);

/* y[c*ldy + r] = sum_k W[r,k] * X[c,k]  for r < n_rows, c < n_cols: the
 * result of ggml's mul_mat for a Q2_K src0 and Q8_K-quantized src1 (dst
 * rows contiguous).  n_rows and k must match the handle.  Up to 15 activation
 * rows run on the decode GEMV, 16 or more on the tensor-core GEMM (the
 * analogue of ggml_gemv_ / ggml_gemm_q2_K_8x8_q8_K); both give identical bits.
 * The GEMM keeps a library-owned device scratch per (device, stream). */
int smeai_q2k_mul_mat(const void *w_dev, int64_t n_rows, int64_t k, const void *x_q8k_dev, int64_t n_cols,
                      float *y_dev, size_t ldy, void *stream);
/* The tensor-core GEMM for any n_cols >= 1 (tcgen05.mma, TMEM accumulators). */
int smeai_q2k_mul_mat_tc(const void *w_dev, const void *x_q8k_dev, int64_t n_cols, float *y_dev, size_t ldy,
                         void *stream);

/* Fused epilogues of the decode GEMV (n_cols <= 8 per launch, larger counts
 * are split):
 *   SMEAI_EPI_STORE     y = W x
 *   SMEAI_EPI_RESIDUAL  y = resid + W x          (resid may alias y)
 *   SMEAI_EPI_SILU_MUL  rows of W interleave (gate_i, up_i);
 *                       y[i] = silu(gate_i . x) * (up_i . x)   (n_rows/2 outputs) */
#define SMEAI_EPI_STORE 0
#define SMEAI_EPI_RESIDUAL 1
#define SMEAI_EPI_SILU_MUL 2
int smeai_q2k_mul_mat_ex(const void *w_dev, const void *x_q8k_dev, int64_t n_cols, float *y_dev, size_t ldy,
                         int epilogue, const float *resid_dev, size_t ld_resid, void *stream);
/* The same epilogues on the tensor-core GEMM (any n_cols >= 1; the prefill
 * path): bit-identical to smeai_q2k_mul_mat_ex on the same inputs. */
int smeai_q2k_mul_mat_tc_ex(const void *w_dev, const void *x_q8k_dev, int64_t n_cols, float *y_dev, size_t ldy,
                            int epilogue, const float *resid_dev, size_t ld_resid, void *stream);

/* ---- decode program: a chain of dependent GEMVs as ONE persistent kernel ----
 * Phase p reads the complete output of phase p-1 (its input buffer is, or
 * contains, that output); each phase is one smeai_q2k_mul_mat_ex /
 * smeai_q2k_mul_mat_f32_ex call and gives the same bits.  One CTA per SM
 * streams every phase's weights back to back; each finished output value is
 * published as one 8-byte tagged word (value + launch tag) that the next
 * phase's warps poll block by block, so a decode step is one launch instead
 * of one per linear (ggml's graph of MUL_MAT nodes over a layer stack, run
 * as a single kernel).  n_cols (tokens) is 1, 2, 4 or 8.
 * The launch is cooperative; a run that hits a bounded-wait timeout (never
 * expected; reported by smeai_take_device_error) needs
 * smeai_q2k_program_reset before the next run. */
#define SMEAI_IN_Q8K 0     /* x: contiguous Q8_K rows */
#define SMEAI_IN_F32 1     /* x: fp32 rows (stride ld_x), quantized to Q8_K in the kernel */
#define SMEAI_IN_F32_RMS 2 /* the same after an RMSNorm of each row (rms_eps) */
typedef struct smeai_q2k_phase {
  const void *w;       /* handle from smeai_q2k_repack */
  int input;           /* SMEAI_IN_* */
  const void *x;
  size_t ld_x;
  float *y;
  size_t ldy;
  int epilogue;        /* SMEAI_EPI_* */
  const float *resid;  /* SMEAI_EPI_RESIDUAL; may alias y */
  size_t ld_resid;
  const float *norm_w; /* SMEAI_IN_F32_RMS: RMSNorm weight (k floats), or NULL */
} smeai_q2k_phase;
int smeai_q2k_program_create(const smeai_q2k_phase *phases, int n_phases, int64_t n_cols, float rms_eps,
                             void **prog_out);

/* The decode program over the row shards of several GPUs of one node (one
 * process and one program per GPU; row-sharded ggml weights, replicated
 * activations).  The phases are wired explicitly: phase p reads rows
 * x_row0.. of phase x_src's GLOBAL output (all ranks' rows), or, with
 * x_src = -1, an outside input x (full rows, replicated on every rank);
 * its local output rows [ex_lo, ex_hi) are global rows ex_row0.. of its own
 * output.  Each finished row is stored, in the kernel that computes it, as a
 * tagged word into every rank's copy of that output over NVLink peer memory
 * (no collective library, no per-phase barrier: a rank starts a phase's
 * block as soon as the words it needs carry the launch's tag).  y receives
 * the local rows.  After create, every rank exports its handle, the ranks
 * swap them (rank order) and connect; then run() on every rank runs a step,
 * and gather() turns a phase's global output into plain floats.  The bounded
 * waits use the peer limit (smeai_set_wait_timeouts).  Bit-identical to the
 * one-GPU program on the unsharded weights. */
typedef struct smeai_q2k_mg_phase {
  const void *w;        /* this rank's row shard (smeai_q2k_repack handle) */
  int input;            /* SMEAI_IN_F32 or SMEAI_IN_F32_RMS */
  int x_src;            /* producing phase, or -1: outside input x */
  int64_t x_row0;
  const float *x;
  size_t ld_x;
  int epilogue;         /* SMEAI_EPI_* */
  int resid_src;        /* residual: rows resid_row0.. of phase resid_src's output, or -1: */
  int64_t resid_row0;   /*   outside resid[t * ld_resid + resid_row0 + r] for local row r */
  const float *resid;
  size_t ld_resid;
  const float *norm_w;  /* RMSNorm weight (SMEAI_IN_F32_RMS), or NULL */
  int64_t out_rows;     /* rows of the global output */
  int64_t ex_lo, ex_hi, ex_row0;
  float *y;
  size_t ldy;
} smeai_q2k_mg_phase;
int smeai_q2k_mg_program_create(const smeai_q2k_mg_phase *phases, int n_phases, int64_t n_cols, float rms_eps,
                                int rank, int world, void **prog_out);
int smeai_q2k_program_ipc_handle(void *prog, void *handle64);
int smeai_q2k_program_connect(void *prog, const void *handles, int world);
int smeai_q2k_program_gather(void *prog, int phase, float *y_dev, size_t ldy, void *stream);
int smeai_q2k_program_run(void *prog, void *stream);
int smeai_q2k_program_reset(void *prog, void *stream);
void smeai_q2k_program_free(void *prog);

/* fp32 activations in, fp32 out: each CTA quantizes the activation rows to
 * Q8_K in its prologue (bit-identical to smeai_q8k_quantize), then runs the
 * GEMV -- one kernel, no intermediate buffer.  x: n_cols rows of k floats. */
int smeai_q2k_mul_mat_f32(const void *w_dev, const float *x_dev, int64_t n_cols, float *y_dev, size_t ldy,
                          void *stream);
/* The same with a row stride, the fused epilogues, and an optional RMSNorm of
 * each activation row before quantization (rms_eps >= 0; < 0 disables it),
 * bit-identical to smeai_rms_q8k_quantize followed by smeai_q2k_mul_mat_ex. */
int smeai_q2k_mul_mat_f32_ex(const void *w_dev, const float *x_dev, size_t ld_x, int64_t n_cols, float *y_dev,
                             size_t ldy, int epilogue, const float *resid_dev, size_t ld_resid, float rms_eps,
                             void *stream);
/* The same with an RMSNorm weight (k floats on the device, NULL = none; needs
 * rms_eps >= 0): bit-identical to smeai_rms_q8k_quantize_w followed by
 * smeai_q2k_mul_mat_ex. */
int smeai_q2k_mul_mat_f32_norm(const void *w_dev, const float *x_dev, size_t ld_x, int64_t n_cols, float *y_dev,
                               size_t ldy, int epilogue, const float *resid_dev, size_t ld_resid, float rms_eps,
                               const float *norm_w_dev, void *stream);

/* Row-sharded GEMV with its all-gather fused in (multi-GPU decode, one process
 * per GPU).  Each rank holds a row shard of W; this call computes the shard's
 * rows like smeai_q2k_mul_mat_f32_ex and, in the same kernel, stores the rows
 * at or past local output row `row0` of every finished 32-row group into each
 * dst[q] (peer memory opened with smeai_ipc_open, or this GPU's own) at row
 * (r - row0), token stride ld_dst floats; when all of a CTA's groups are
 * stored it raises each sig[q] by its number of row groups (system-scope
 * fence, then the additions), so every row group of the call counts once.  When wait_sig is set the kernel first waits (bounded,
 * 10 s; a timeout is reported by smeai_take_device_error) until *wait_sig has
 * reached (*epoch + 1) * wait_count -- the row groups every rank of the
 * producing call publishes per step -- so its input may be rows other GPUs
 * store.  n_cols must be 1, 2, 4 or 8 (one launch); Q2_K weights, fp32 input. */
typedef struct {
    int n_dst;                  /* destinations (<= 8) */
    float *dst[8];
    int64_t ld_dst;
    int64_t row0;               /* first exchanged local output row (a multiple of 16) */
    int n_sig;                  /* signal words bumped per exchanged row group (<= 8) */
    unsigned *sig[8];
    const unsigned *wait_sig;   /* NULL: no wait */
    unsigned wait_count;
    const unsigned *epoch;      /* this rank's step counter (device word) */
} smeai_peer_exchange;
int smeai_q2k_mul_mat_f32_peer(const void *w_dev, const float *x_dev, size_t ld_x, int64_t n_cols, float *y_dev,
                               size_t ldy, int epilogue, const float *resid_dev, size_t ld_resid, float rms_eps,
                               const float *norm_w_dev, const smeai_peer_exchange *ex, void *stream);
/* End of a step: wait (bounded) until *sig reaches (*epoch + 1) * count, then
 * advance *epoch (queued on stream; one thread). */
int smeai_peer_step_end(const unsigned *sig, unsigned count, unsigned *epoch, void *stream);
/* Device memory shareable with the other processes of the node: bytes
 * zero-filled, *ptr its address here, handle[64] the CUDA IPC handle to send
 * to the peers, which map it with smeai_ipc_open (peer access enabled). */
int smeai_ipc_alloc(size_t bytes, void **ptr, void *handle64);
void smeai_ipc_free(void *ptr);
int smeai_ipc_open(const void *handle64, void **ptr);
void smeai_ipc_close(void *ptr);

/* Exactness probe: the integer parts of the dot for every (row, super-block)
 * against ONE Q8_K row, [n_rows][k/256] int32 each:
 *   isum  = sum_j scale_j * sum_{i in sub-block j} q2_i * q8_i
 *   summs = sum_j min_j * bsums_j                                          */
int smeai_q2k_block_sums(const void *w_dev, const void *x_q8k_dev, int32_t *isum_dev, int32_t *summs_dev,
                         void *stream);

/* Device-side weight quantizer / decoder (fp32 <-> block_q2_K, n % 256 == 0). */
int smeai_q2k_quantize_device(const float *x_dev, int64_t n, void *y_q2k_dev, void *stream);
int smeai_q2k_dequantize_device(const void *w_q2k_dev, int64_t n, float *y_dev, void *stream);

/* ---------------- 3. Q3_K weights ----------------------------------------
 * The reference leaves its Q3_K tensors (110 of the TinyLlama Q2_K file's 201,
 * llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:44-51) on ggml's generic path; these
 * are that path's entry points on the GPU.  block_q3_K = hmask[32] qs[64]
 * scales[12] d(fp16) = 110 bytes per 256 weights.  The per-super-block
 * integer sums equal ggml's exactly; ggml's generic dot then accumulates
 * floats in 8 position lanes, the GPU in one (ascending super-blocks), so
 * outputs agree to float rounding (reordered accumulation). */

/* ggml type-trait shapes (host pointers; see group 1 above). */
void dequantize_row_q3_K(const void *x, float *y, int64_t k);
void ggml_vec_dot_q3_K_q8_K(int n, float *s, size_t bs, const void *vx, size_t bx, const void *vy, size_t by,
                            int nrc);

/* Repack n_rows x k of block_q3_K (host or device) into the device tile
 * layout; the handle is freed with smeai_q3k_free (or smeai_q2k_free). */
int smeai_q3k_repack(const void *w_q3k, int64_t n_rows, int64_t k, void **w_dev_out);
void smeai_q3k_free(void *w_dev);
/* y[c*ldy + r] = row r . activation c for n_cols Q8_K rows (device). */
int smeai_q3k_mul_mat(const void *w_dev, const void *x_q8k_dev, int64_t n_cols, float *y_dev, size_t ldy,
                      void *stream);
/* The same from fp32 activation rows (stride ld_x floats), quantized to Q8_K
 * inside the kernel, after an RMSNorm when rms_eps >= 0. */
int smeai_q3k_mul_mat_f32(const void *w_dev, const float *x_dev, size_t ld_x, int64_t n_cols, float *y_dev,
                          size_t ldy, float rms_eps, void *stream);
/* Per-(row, super-block) integer sums for one activation row: isum (ggml's
 * integer total) and summs = sum_j (scale_j - 32) * bsums_j, [n_rows][nb]. */
int smeai_q3k_block_sums(const void *w_dev, const void *x_q8k_dev, int32_t *isum_dev, int32_t *summs_dev,
                         void *stream);
/* Device decode of n weights (n/256 blocks) to fp32. */
int smeai_q3k_dequantize_device(const void *w_q3k_dev, int64_t n, float *y_dev, void *stream);

/* ---------------- 4. Q6_K weights ----------------------------------------
 * The reference model's one Q6_K tensor (llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:
 * 44-51) on ggml's generic path.  block_q6_K = ql[128] qh[64] scales[16]
 * (int8) d(fp16) = 210 bytes per 256 weights.  Same contract as Q3_K: the
 * per-super-block integers equal ggml's; ggml accumulates floats in 8
 * position lanes, the GPU in one. */
void dequantize_row_q6_K(const void *x, float *y, int64_t k);
void ggml_vec_dot_q6_K_q8_K(int n, float *s, size_t bs, const void *vx, size_t bx, const void *vy, size_t by,
                            int nrc);
int smeai_q6k_repack(const void *w_q6k, int64_t n_rows, int64_t k, void **w_dev_out);
void smeai_q6k_free(void *w_dev);
int smeai_q6k_mul_mat(const void *w_dev, const void *x_q8k_dev, int64_t n_cols, float *y_dev, size_t ldy,
                      void *stream);
int smeai_q6k_mul_mat_f32(const void *w_dev, const float *x_dev, size_t ld_x, int64_t n_cols, float *y_dev,
                          size_t ldy, float rms_eps, void *stream);
/* isum (ggml's integer total) and summs = sum_j scale_j * bsums_j. */
int smeai_q6k_block_sums(const void *w_dev, const void *x_q8k_dev, int32_t *isum_dev, int32_t *summs_dev,
                         void *stream);
int smeai_q6k_dequantize_device(const void *w_q6k_dev, int64_t n, float *y_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif
