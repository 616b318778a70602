// kernels.h -- host-side launchers of the sm_100a kernels (internal to the
// library; the public C entry points live in include/*.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace smeai {

// ---- Q8_K activation quantizer (q8k_quant.cu) ----
int q8k_quantize(const float* x, int64_t ld_x, int64_t n_rows, int64_t k, void* y, cudaStream_t stream);
// RMSNorm of each row (times norm_w[k] when norm_w is not null, the
// reference's weight operand), then Q8_K.
int rms_q8k_quantize(const float* x, int64_t ld_x, int64_t n_rows, int64_t k, float eps, void* y,
                     cudaStream_t stream, const float* norm_w = nullptr);

// ---- Q2_K weight quantizer / decoder (q2k_quant.cu) ----
int q2k_quantize(const float* x, int64_t k_total, void* y, cudaStream_t stream);
int q2k_dequantize(const void* w, int64_t k_total, float* y, cudaStream_t stream);

// ---- Q2_K weights in the device tile layout (q2k_gemv.cu) ----
// Rows are grouped by 32; group g, super-block b is one 2688-byte tile:
//   qs     4 x [32 rows][16 B]   (chunk c holds qs bytes 16c..16c+15)
//   scales    [32 rows][16 B]
//   d,dmin    [32 rows][4 B]
constexpr int kRowsPerGroup = 32;
constexpr int kTileBytes = 32 * 84;

// Weight formats held in the tile layout (tile bytes per 32-row group and
// super-block: Q2_K 2688, Q3_K 3584 -- see q3k_core.cuh).
enum WeightFmt : int { kFmtQ2K = 0, kFmtQ3K = 1, kFmtQ6K = 2 };
// Tile bytes per (32-row group, super-block) of each format.
inline int fmt_tile_bytes(int fmt) { return fmt == kFmtQ3K ? 32 * 112 : fmt == kFmtQ6K ? 32 * 212 : 32 * 84; }

struct Q2KWeight {
  int fmt = kFmtQ2K;
  int64_t n_rows = 0;
  int64_t k = 0;
  int nb = 0;           // super-blocks per row
  int64_t n_groups = 0; // ceil(n_rows / 32)
  uint8_t* tiles = nullptr;  // device, n_groups * nb * kTileBytes
  size_t bytes = 0;
  int device = 0;
};

int q2k_repack(const void* w_blocks_dev, int64_t n_rows, int64_t k, Q2KWeight* out, cudaStream_t stream);
// Same, into caller-provided tiles (tile_bytes(n_rows, k) bytes); allocates nothing.
size_t q2k_tile_bytes(int64_t n_rows, int64_t k);
int q2k_repack_into(const void* w_blocks_dev, int64_t n_rows, int64_t k, uint8_t* tiles, Q2KWeight* out,
                    cudaStream_t stream);

// ---- Q3_K weights (q3k_quant.cu): ggml blocks -> tiles, decode ----
size_t q3k_tile_bytes(int64_t n_rows, int64_t k);
int q3k_repack_into(const void* w_blocks_dev, int64_t n_rows, int64_t k, uint8_t* tiles, Q2KWeight* out,
                    cudaStream_t stream);
int q3k_repack(const void* w_blocks_dev, int64_t n_rows, int64_t k, Q2KWeight* out, cudaStream_t stream);
int q3k_dequantize(const void* w, int64_t k_total, float* y, cudaStream_t stream);

// ---- Q6_K weights (q6k_quant.cu) ----
size_t q6k_tile_bytes(int64_t n_rows, int64_t k);
int q6k_repack_into(const void* w_blocks_dev, int64_t n_rows, int64_t k, uint8_t* tiles, Q2KWeight* out,
                    cudaStream_t stream);
int q6k_repack(const void* w_blocks_dev, int64_t n_rows, int64_t k, Q2KWeight* out, cudaStream_t stream);
int q6k_dequantize(const void* w, int64_t k_total, float* y, cudaStream_t stream);

enum Epilogue : int {
  kEpiStore = 0,     // y[c*ldy + r] = acc
  kEpiResidual = 1,  // y[c*ldy + r] = resid[c*ld_resid + r] + acc   (resid may alias y)
  kEpiSiluMul = 2,   // rows interleaved (gate, up): y[c*ldy + r/2] = silu(gate) * up
};

// Activation input of the GEMV: ggml Q8_K blocks (contiguous rows), or fp32
// rows quantized to Q8_K in the kernel's prologue, optionally after an RMSNorm.
enum InMode : int { kInQ8K = 0, kInF32 = 1, kInF32Rms = 2 };

// Cross-GPU exchange of a row-sharded GEMV's output (peer memory mapped
// through CUDA IPC): the rows of every finished row group at or past local
// output row row0 are also stored to each dst[q] (at row - row0, token stride
// ld_dst); once all of a CTA's groups are stored, each sig[q] is raised by
// the CTA's number of row groups (one system-scope fence, then relaxed
// reductions) -- so a full count also says that every CTA of the call has
// finished reading its input.  A GEMV with
// wait_sig first waits (bounded) until *wait_sig reaches
// (*epoch + 1) * wait_count -- every rank's row groups of the producing GEMV in
// this step -- and then reads its input through L2.
constexpr int kMaxPeers = 8;
struct PeerExchange {
  int n_dst = 0;
  float* dst[kMaxPeers] = {};
  int64_t ld_dst = 0;
  int64_t row0 = 0;
  int n_sig = 0;
  unsigned* sig[kMaxPeers] = {};
  const unsigned* wait_sig = nullptr;
  unsigned wait_count = 0;
  const unsigned* epoch = nullptr;
};

// norm_w: the RMSNorm weight of a kInF32Rms input (null: none).
int q2k_gemv_any(const Q2KWeight& w, int in_mode, const void* x, int64_t ld_x, float eps, int64_t n_cols,
                 float* y, int64_t ldy, int epilogue, const float* resid, int64_t ld_resid, cudaStream_t stream,
                 const PeerExchange* ex = nullptr, const float* norm_w = nullptr);
// End of a step on one rank: wait (bounded) until *sig reaches
// (*epoch + 1) * count, then advance *epoch.
int peer_step_end(const unsigned* sig, unsigned count, unsigned* epoch, cudaStream_t stream);

// y = W x for n_cols Q8_K activation rows (ggml layout, contiguous rows).
int q2k_gemv(const Q2KWeight& w, const void* xq, int64_t n_cols, float* y, int64_t ldy, int epilogue,
             const float* resid, int64_t ld_resid, cudaStream_t stream);

// A decode step as one persistent cooperative kernel (q2k_program.cu): the
// phases run in order, phase p reading the complete output of phase p-1;
// every output is bit-identical to running the phases as separate q2k_gemv_any
// launches (same input modes, epilogues and quantizers).
struct ProgPhase {
  const Q2KWeight* w = nullptr;
  int in_mode = kInQ8K;        // kInQ8K: x = contiguous Q8_K rows; kInF32 / kInF32Rms: fp32 rows
  const void* x = nullptr;
  int64_t ld_x = 0;            // fp32 row stride (floats)
  float* y = nullptr;
  int64_t ldy = 0;
  int epi = kEpiStore;
  const float* resid = nullptr;
  int64_t ld_resid = 0;
  const float* norm_w = nullptr;  // RMSNorm weight of a kInF32Rms input (null: none)
};
struct Q2KProgram;
int q2k_program_create(const ProgPhase* phases, int n_phases, int n_cols, float rms_eps, Q2KProgram** out);
// The same over the row shards of several GPUs (one program per rank), with
// the phases wired explicitly: a phase reads rows x_row0.. of phase x_src's
// global output (or an outside input x replicated on every rank), and stores
// its local output rows [ex_lo, ex_hi) as global rows ex_row0.. of its own
// output -- into every rank's copy, over peer memory.
struct MGPhase {
  const Q2KWeight* w = nullptr;
  int in_mode = kInF32;
  int x_src = -1;
  int64_t x_row0 = 0;
  const float* x = nullptr;
  int64_t ld_x = 0;
  int epi = kEpiStore;
  int r_src = -1;           // residual: rows r_row0.. of phase r_src's global output, or outside
  int64_t r_row0 = 0;       //   (outside: resid[t * ld_resid + r_row0 + r] for local row r)
  const float* resid = nullptr;
  int64_t ld_resid = 0;
  const float* norm_w = nullptr;
  int64_t out_rows = 0;     // rows of the global output
  int64_t ex_lo = 0, ex_hi = 0, ex_row0 = 0;
  float* y = nullptr;       // this rank's local output rows
  int64_t ldy = 0;
};
int q2k_mg_program_create(const MGPhase* phases, int n_phases, int n_cols, float rms_eps, int rank, int world,
                          Q2KProgram** out);
// Multi-GPU: this rank's IPC handle of its tagged buffers (64 bytes), and the
// mapping of every rank's buffers from the handles of all ranks (rank order).
int q2k_program_ipc_handle(Q2KProgram* prog, void* handle64);
int q2k_program_connect(Q2KProgram* prog, const void* handles, int world);
// After a run: a phase's global output (all ranks' rows) as plain floats.
int q2k_program_gather(Q2KProgram* prog, int phase, float* y, int64_t ldy, cudaStream_t stream);
int q2k_program_run(Q2KProgram* prog, cudaStream_t stream);
int q2k_program_reset(Q2KProgram* prog, cudaStream_t stream);
void q2k_program_free(Q2KProgram* prog);
void q2k_program_shape(const Q2KProgram* prog, int* grid, int* consumers, int* stages, size_t* smem);

// Tensor-core GEMM for many activation rows (prefill): y = W x for n_cols
// Q8_K rows, store epilogue, bit-identical to q2k_gemv.  Needs a 256-byte
// aligned scratch of q2k_gemm_scratch_bytes(n_cols, nb) bytes.
size_t q2k_gemm_scratch_bytes(int64_t n_cols, int nb);
// epi: kEpiStore, kEpiResidual (y = resid + W x; resid may alias y) or
// kEpiSiluMul (rows interleave gate/up; y gets n_rows / 2 values per token),
// the arithmetic of the GEMV's epilogues.
int q2k_gemm_tc(const Q2KWeight& w, const void* xq, int64_t n_cols, float* y, int64_t ldy, void* scratch,
                size_t scratch_bytes, cudaStream_t stream, int epi = kEpiStore, const float* resid = nullptr,
                int64_t ld_resid = 0);

// Per-(row, super-block) integer sums (isum, summs), [n_rows][nb] each, for a
// single activation row -- the exactness check of the GEMV's integer core.
int q2k_block_sums(const Q2KWeight& w, const void* xq, int32_t* isum, int32_t* summs, cudaStream_t stream);

}  // namespace smeai
