// api_q2k.cu -- the C-ABI of include/smeai_q2k.h.
#include <string.h>

#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "runtime.h"
#include "../../include/smeai_q2k.h"

using namespace smeai;

namespace {

constexpr uint32_t kHandleMagic = 0x51324b57u;  // "Q2KW"
constexpr int64_t kQ3KBytes = 110;               // ggml block_q3_K
constexpr int64_t kQ6KBytes = 210;               // ggml block_q6_K

struct Handle {
  uint32_t magic = kHandleMagic;
  Q2KWeight w;
};

const Handle* as_handle(const void* p) {
  const Handle* h = static_cast<const Handle*>(p);
  if (!h || h->magic != kHandleMagic) {
    set_last_error("not a repacked weight handle");
    return nullptr;
  }
  return h;
}

// A handle of the given weight format (Q2_K entry points refuse Q3_K handles
// and the reverse).
const Handle* as_fmt(const void* p, int fmt, const char* what) {
  const Handle* h = as_handle(p);
  if (h && h->w.fmt != fmt) {
    set_last_error("%s: the handle holds a %s weight", what,
                   h->w.fmt == kFmtQ3K ? "Q3_K" : h->w.fmt == kFmtQ6K ? "Q6_K" : "Q2_K");
    return nullptr;
  }
  return h;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Per-thread state of the ggml-shaped entry points: own stream + staging.
struct ThreadCtx {
  cudaStream_t stream = nullptr;
  Staged a, b;
  DeviceBuffer tiles, y;
  int init() {
    if (stream) return kOk;
    SMEAI_CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    return kOk;
  }
};

ThreadCtx& tctx() {
  thread_local ThreadCtx ctx;
  return ctx;
}

// Library-owned scratch of the tensor-core GEMM (activation operands in UMMA
// order), one growable buffer per (device, stream).
std::mutex g_gemm_mu;
std::map<std::pair<int, cudaStream_t>, DeviceBuffer*> g_gemm_scratch;

int gemm_scratch(cudaStream_t s, size_t bytes, void** out) {
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_gemm_mu);
  DeviceBuffer*& b = g_gemm_scratch[{dev, s}];
  if (!b) b = new DeviceBuffer();
  const int st = b->reserve(bytes);
  if (st) return st;
  *out = b->ptr;
  return kOk;
}

// Activation rows at which mul_mat switches from the GEMV to the tensor cores.
constexpr int64_t kGemmMinCols = 16;

int mul_mat_tc(const Q2KWeight& w, const void* xq, int64_t n_cols, float* y, int64_t ldy, cudaStream_t s,
               int epi = kEpiStore, const float* resid = nullptr, int64_t ld_resid = 0) {
  const size_t need = q2k_gemm_scratch_bytes(n_cols, w.nb);
  void* scratch = nullptr;
  const int st = gemm_scratch(s, need, &scratch);
  if (st) return st;
  return q2k_gemm_tc(w, xq, n_cols, y, ldy, scratch, need, s, epi, resid, ld_resid);
}

}  // namespace

extern "C" {

int smeai_device_ready(void) { return device_ready() ? 1 : 0; }

const char* smeai_last_error(void) { return last_error(); }

int smeai_take_device_error(unsigned* code) {
  if (!code) {
    set_last_error("smeai_take_device_error: NULL pointer");
    return kBadArgument;
  }
  return device_error_take(code);
}

void smeai_set_wait_timeouts(uint64_t local_ns, uint64_t peer_ns) { set_wait_timeouts(local_ns, peer_ns); }

void smeai_debug_fail_next_allocs(int n) { fail_next_allocs(n); }

// ---- ggml-shaped entry points ------------------------------------------------

void quantize_row_q8_K(const float* x, void* y, int64_t k) {
  if (!x || !y || k <= 0 || k % QK_K) {
    set_last_error("quantize_row_q8_K: k must be a positive multiple of 256");
    return;
  }
  ThreadCtx& c = tctx();
  const size_t out_bytes = (size_t)(k / QK_K) * Q8K_BLOCK_BYTES;
  if (c.init() || c.a.in(x, (size_t)k * 4, c.stream) || c.b.out(y, out_bytes) ||
      q8k_quantize(static_cast<const float*>(c.a.dev), k, 1, k, c.b.dev, c.stream) || c.b.finish(c.stream) ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    if (!is_device_pointer(y)) memset(y, 0, out_bytes);
  }
}

void quantize_row_q2_K(const float* x, void* y, int64_t k) {
  if (!x || !y || k <= 0 || k % QK_K) {
    set_last_error("quantize_row_q2_K: k must be a positive multiple of 256");
    return;
  }
  ThreadCtx& c = tctx();
  const size_t out_bytes = (size_t)(k / QK_K) * Q2K_BLOCK_BYTES;
  if (c.init() || c.a.in(x, (size_t)k * 4, c.stream) || c.b.out(y, out_bytes) ||
      q2k_quantize(static_cast<const float*>(c.a.dev), k, c.b.dev, c.stream) || c.b.finish(c.stream) ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    if (!is_device_pointer(y)) memset(y, 0, out_bytes);
  }
}

void dequantize_row_q2_K(const void* x, float* y, int64_t k) {
  if (!x || !y || k <= 0 || k % QK_K) {
    set_last_error("dequantize_row_q2_K: k must be a positive multiple of 256");
    return;
  }
  ThreadCtx& c = tctx();
  if (c.init() || c.a.in(x, (size_t)(k / QK_K) * Q2K_BLOCK_BYTES, c.stream) || c.b.out(y, (size_t)k * 4) ||
      q2k_dequantize(c.a.dev, k, static_cast<float*>(c.b.dev), c.stream) || c.b.finish(c.stream) ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    if (!is_device_pointer(y)) memset(y, 0, (size_t)k * 4);
  }
}

void ggml_vec_dot_q2_K_q8_K(int n, float* s, size_t bs, const void* vx, size_t bx, const void* vy, size_t by,
                            int nrc) {
  (void)bs;
  (void)bx;
  (void)by;
  if (!s) return;
  *s = 0.f;
  if (!vx || !vy || n <= 0 || n % QK_K || nrc != 1) {
    set_last_error("ggml_vec_dot_q2_K_q8_K: needs n %% 256 == 0 and nrc == 1");
    return;
  }
  ThreadCtx& c = tctx();
  const int64_t nb = n / QK_K;
  Q2KWeight w;
  if (c.init() || c.a.in(vx, nb * Q2K_BLOCK_BYTES, c.stream) || c.b.in(vy, nb * Q8K_BLOCK_BYTES, c.stream) ||
      c.tiles.reserve(q2k_tile_bytes(1, n)) || c.y.reserve(4) ||
      q2k_repack_into(c.a.dev, 1, n, static_cast<uint8_t*>(c.tiles.ptr), &w, c.stream) ||
      q2k_gemv(w, c.b.dev, 1, static_cast<float*>(c.y.ptr), 1, kEpiStore, nullptr, 0, c.stream) ||
      cudaMemcpyAsync(s, c.y.ptr, 4, cudaMemcpyDeviceToHost, c.stream) != cudaSuccess ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    *s = 0.f;
  }
}

// ---- coarse GPU entry points ---------------------------------------------------

int smeai_q2k_repack(const void* w_q2k, int64_t n_rows, int64_t k, void** w_dev_out) {
  if (!w_q2k || !w_dev_out || n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("smeai_q2k_repack: bad arguments");
    return kBadArgument;
  }
  *w_dev_out = nullptr;
  if (!device_ready()) {
    set_last_error("smeai_q2k_repack: no compute-capability-10.x device");
    return kUnsupported;
  }
  Staged src;
  const size_t bytes = (size_t)n_rows * (size_t)(k / QK_K) * Q2K_BLOCK_BYTES;
  int st = src.in(w_q2k, bytes, nullptr);
  if (st) return st;
  Handle* h = new Handle();
  st = q2k_repack(src.dev, n_rows, k, &h->w, nullptr);
  if (st == kOk && cudaStreamSynchronize(nullptr) != cudaSuccess) {
    set_last_error("smeai_q2k_repack: %s", cudaGetErrorString(cudaGetLastError()));
    st = kCudaError;
  }
  if (st) {
    if (h->w.tiles) cudaFree(h->w.tiles);
    delete h;
    return st;
  }
  *w_dev_out = h;
  return kOk;
}

void smeai_q2k_free(void* w_dev) {
  Handle* h = static_cast<Handle*>(w_dev);
  if (!h || h->magic != kHandleMagic) return;
  if (h->w.tiles) cudaFree(h->w.tiles);
  h->magic = 0;
  delete h;
}

size_t smeai_q2k_weight_bytes(const void* w_dev) {
  const Handle* h = as_handle(w_dev);
  return h ? h->w.bytes : 0;
}

int smeai_q8k_quantize(const float* x_dev, int64_t ld_x, int64_t n_cols, int64_t k, void* y_q8k_dev,
                       void* stream) {
  if (!x_dev || !y_q8k_dev) {
    set_last_error("smeai_q8k_quantize: NULL pointer");
    return kBadArgument;
  }
  return q8k_quantize(x_dev, ld_x, n_cols, k, y_q8k_dev, as_stream(stream));
}

int smeai_rms_q8k_quantize(const float* x_dev, int64_t ld_x, int64_t n_cols, int64_t k, float eps,
                           void* y_q8k_dev, void* stream) {
  if (!x_dev || !y_q8k_dev) {
    set_last_error("smeai_rms_q8k_quantize: NULL pointer");
    return kBadArgument;
  }
  return rms_q8k_quantize(x_dev, ld_x, n_cols, k, eps, y_q8k_dev, as_stream(stream));
}

int smeai_rms_q8k_quantize_w(const float* x_dev, int64_t ld_x, int64_t n_cols, int64_t k, const float* weight_dev,
                             float eps, void* y_q8k_dev, void* stream) {
  if (!x_dev || !y_q8k_dev) {
    set_last_error("smeai_rms_q8k_quantize_w: NULL pointer");
    return kBadArgument;
  }
  return rms_q8k_quantize(x_dev, ld_x, n_cols, k, eps, y_q8k_dev, as_stream(stream), weight_dev);
}

int smeai_q2k_mul_mat(const void* w_dev, int64_t n_rows, int64_t k, const void* x_q8k_dev, int64_t n_cols,
                      float* y_dev, size_t ldy, void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_mul_mat");
  if (!h) return kBadArgument;
  if (h->w.n_rows != n_rows || h->w.k != k) {
    set_last_error("smeai_q2k_mul_mat: shape [%lld,%lld] does not match the handle [%lld,%lld]",
                   (long long)n_rows, (long long)k, (long long)h->w.n_rows, (long long)h->w.k);
    return kBadArgument;
  }
  if (n_cols >= kGemmMinCols) return mul_mat_tc(h->w, x_q8k_dev, n_cols, y_dev, (int64_t)ldy, as_stream(stream));
  return q2k_gemv(h->w, x_q8k_dev, n_cols, y_dev, (int64_t)ldy, kEpiStore, nullptr, 0, as_stream(stream));
}

int smeai_q2k_mul_mat_tc(const void* w_dev, const void* x_q8k_dev, int64_t n_cols, float* y_dev, size_t ldy,
                         void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_mul_mat_tc");
  if (!h) return kBadArgument;
  return mul_mat_tc(h->w, x_q8k_dev, n_cols, y_dev, (int64_t)ldy, as_stream(stream));
}

int smeai_q2k_mul_mat_tc_ex(const void* w_dev, const void* x_q8k_dev, int64_t n_cols, float* y_dev, size_t ldy,
                            int epilogue, const float* resid_dev, size_t ld_resid, void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_mul_mat_tc_ex");
  if (!h) return kBadArgument;
  return mul_mat_tc(h->w, x_q8k_dev, n_cols, y_dev, (int64_t)ldy, as_stream(stream), epilogue, resid_dev,
                    (int64_t)ld_resid);
}

int smeai_q2k_mul_mat_ex(const void* w_dev, const void* x_q8k_dev, int64_t n_cols, float* y_dev, size_t ldy,
                         int epilogue, const float* resid_dev, size_t ld_resid, void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_mul_mat_ex");
  if (!h) return kBadArgument;
  return q2k_gemv(h->w, x_q8k_dev, n_cols, y_dev, (int64_t)ldy, epilogue, resid_dev, (int64_t)ld_resid,
                  as_stream(stream));
}

int smeai_q2k_program_create(const smeai_q2k_phase* phases, int n_phases, int64_t n_cols, float rms_eps,
                             void** prog_out) {
  if (!phases || !prog_out || n_phases <= 0 || n_cols <= 0 || n_cols > 8) {
    set_last_error("smeai_q2k_program_create: bad arguments");
    return kBadArgument;
  }
  *prog_out = nullptr;
  std::vector<ProgPhase> ph((size_t)n_phases);
  for (int p = 0; p < n_phases; ++p) {
    const Handle* h = as_fmt(phases[p].w, kFmtQ2K, "smeai_q2k_program_create");
    if (!h) return kBadArgument;
    ProgPhase& d = ph[(size_t)p];
    d.w = &h->w;
    d.in_mode = phases[p].input;
    d.x = phases[p].x;
    d.ld_x = (int64_t)phases[p].ld_x;
    d.y = phases[p].y;
    d.ldy = (int64_t)phases[p].ldy;
    d.epi = phases[p].epilogue;
    d.resid = phases[p].resid;
    d.ld_resid = (int64_t)phases[p].ld_resid;
    d.norm_w = phases[p].norm_w;
  }
  Q2KProgram* pr = nullptr;
  const int st = q2k_program_create(ph.data(), n_phases, (int)n_cols, rms_eps, &pr);
  if (st == kOk) *prog_out = pr;
  return st;
}

int smeai_q2k_mg_program_create(const smeai_q2k_mg_phase* phases, int n_phases, int64_t n_cols, float rms_eps,
                                int rank, int world, void** prog_out) {
  if (!phases || !prog_out || n_phases <= 0 || n_cols <= 0 || n_cols > 8) {
    set_last_error("smeai_q2k_mg_program_create: bad arguments");
    return kBadArgument;
  }
  *prog_out = nullptr;
  std::vector<MGPhase> ph((size_t)n_phases);
  for (int p = 0; p < n_phases; ++p) {
    const Handle* h = as_fmt(phases[p].w, kFmtQ2K, "smeai_q2k_mg_program_create");
    if (!h) return kBadArgument;
    const smeai_q2k_mg_phase& s = phases[p];
    MGPhase& d = ph[(size_t)p];
    d.w = &h->w;
    d.in_mode = s.input;
    d.x_src = s.x_src;
    d.x_row0 = s.x_row0;
    d.x = s.x;
    d.ld_x = (int64_t)s.ld_x;
    d.epi = s.epilogue;
    d.r_src = s.resid_src;
    d.r_row0 = s.resid_row0;
    d.resid = s.resid;
    d.ld_resid = (int64_t)s.ld_resid;
    d.norm_w = s.norm_w;
    d.out_rows = s.out_rows;
    d.ex_lo = s.ex_lo;
    d.ex_hi = s.ex_hi;
    d.ex_row0 = s.ex_row0;
    d.y = s.y;
    d.ldy = (int64_t)s.ldy;
  }
  Q2KProgram* pr = nullptr;
  const int st = q2k_mg_program_create(ph.data(), n_phases, (int)n_cols, rms_eps, rank, world, &pr);
  if (st == kOk) *prog_out = pr;
  return st;
}

int smeai_q2k_program_ipc_handle(void* prog, void* handle64) {
  return q2k_program_ipc_handle(static_cast<Q2KProgram*>(prog), handle64);
}

int smeai_q2k_program_connect(void* prog, const void* handles, int world) {
  return q2k_program_connect(static_cast<Q2KProgram*>(prog), handles, world);
}

int smeai_q2k_program_gather(void* prog, int phase, float* y_dev, size_t ldy, void* stream) {
  return q2k_program_gather(static_cast<Q2KProgram*>(prog), phase, y_dev, (int64_t)ldy, as_stream(stream));
}

int smeai_q2k_program_run(void* prog, void* stream) {
  return q2k_program_run(static_cast<Q2KProgram*>(prog), as_stream(stream));
}

int smeai_q2k_program_reset(void* prog, void* stream) {
  return q2k_program_reset(static_cast<Q2KProgram*>(prog), as_stream(stream));
}

void smeai_q2k_program_free(void* prog) { q2k_program_free(static_cast<Q2KProgram*>(prog)); }

int smeai_q2k_mul_mat_f32(const void* w_dev, const float* x_dev, int64_t n_cols, float* y_dev, size_t ldy,
                          void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_mul_mat_f32");
  if (!h) return kBadArgument;
  return q2k_gemv_any(h->w, kInF32, x_dev, h->w.k, 0.f, n_cols, y_dev, (int64_t)ldy, kEpiStore, nullptr, 0,
                      as_stream(stream));
}

int smeai_q2k_mul_mat_f32_ex(const void* w_dev, const float* x_dev, size_t ld_x, int64_t n_cols, float* y_dev,
                             size_t ldy, int epilogue, const float* resid_dev, size_t ld_resid, float rms_eps,
                             void* stream) {
  return smeai_q2k_mul_mat_f32_norm(w_dev, x_dev, ld_x, n_cols, y_dev, ldy, epilogue, resid_dev, ld_resid, rms_eps,
                                    nullptr, stream);
}

int smeai_q2k_mul_mat_f32_norm(const void* w_dev, const float* x_dev, size_t ld_x, int64_t n_cols, float* y_dev,
                               size_t ldy, int epilogue, const float* resid_dev, size_t ld_resid, float rms_eps,
                               const float* norm_w_dev, void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_mul_mat_f32_norm");
  if (!h) return kBadArgument;
  if (norm_w_dev && rms_eps < 0.f) {
    set_last_error("smeai_q2k_mul_mat_f32_norm: an RMSNorm weight needs rms_eps >= 0");
    return kBadArgument;
  }
  return q2k_gemv_any(h->w, rms_eps >= 0.f ? kInF32Rms : kInF32, x_dev, (int64_t)ld_x, rms_eps, n_cols, y_dev,
                      (int64_t)ldy, epilogue, resid_dev, (int64_t)ld_resid, as_stream(stream), nullptr, norm_w_dev);
}

int smeai_q2k_mul_mat_f32_peer(const void* w_dev, const float* x_dev, size_t ld_x, int64_t n_cols, float* y_dev,
                               size_t ldy, int epilogue, const float* resid_dev, size_t ld_resid, float rms_eps,
                               const float* norm_w_dev, const smeai_peer_exchange* ex, void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_mul_mat_f32_peer");
  if (!h) return kBadArgument;
  if (!ex) {
    set_last_error("smeai_q2k_mul_mat_f32_peer: NULL exchange");
    return kBadArgument;
  }
  PeerExchange e;
  e.n_dst = ex->n_dst;
  e.n_sig = ex->n_sig;
  if (e.n_dst < 0 || e.n_dst > kMaxPeers || e.n_sig < 0 || e.n_sig > kMaxPeers) {
    set_last_error("smeai_q2k_mul_mat_f32_peer: at most %d destinations and signals", kMaxPeers);
    return kBadArgument;
  }
  for (int q = 0; q < e.n_dst; ++q) e.dst[q] = ex->dst[q];
  for (int q = 0; q < e.n_sig; ++q) e.sig[q] = ex->sig[q];
  e.ld_dst = ex->ld_dst;
  e.row0 = ex->row0;
  e.wait_sig = ex->wait_sig;
  e.wait_count = ex->wait_count;
  e.epoch = ex->epoch;
  return q2k_gemv_any(h->w, rms_eps >= 0.f ? kInF32Rms : kInF32, x_dev, (int64_t)ld_x, rms_eps, n_cols, y_dev,
                      (int64_t)ldy, epilogue, resid_dev, (int64_t)ld_resid, as_stream(stream), &e, norm_w_dev);
}

int smeai_peer_step_end(const unsigned* sig, unsigned count, unsigned* epoch, void* stream) {
  return peer_step_end(sig, count, epoch, as_stream(stream));
}

int smeai_ipc_alloc(size_t bytes, void** ptr, void* handle64) {
  if (!ptr || !handle64 || !bytes) {
    set_last_error("smeai_ipc_alloc: bad arguments");
    return kBadArgument;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  void* p = nullptr;
  if (device_malloc((void**)&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_last_error("smeai_ipc_alloc: cudaMalloc of %zu bytes failed", bytes);
    return kAllocFailed;
  }
  cudaIpcMemHandle_t hd;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&hd, p) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    cudaFree(p);
    set_last_error("smeai_ipc_alloc: %s", cudaGetErrorString(e));
    return kCudaError;
  }
  memcpy(handle64, &hd, sizeof(hd));
  *ptr = p;
  return kOk;
}

void smeai_ipc_free(void* ptr) {
  if (ptr) cudaFree(ptr);
}

int smeai_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) {
    set_last_error("smeai_ipc_open: bad arguments");
    return kBadArgument;
  }
  cudaIpcMemHandle_t hd;
  memcpy(&hd, handle64, sizeof(hd));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_last_error("smeai_ipc_open: %s", cudaGetErrorString(e));
    return kUnsupported;
  }
  *ptr = p;
  return kOk;
}

void smeai_ipc_close(void* ptr) {
  if (ptr) cudaIpcCloseMemHandle(ptr);
}

int smeai_q2k_block_sums(const void* w_dev, const void* x_q8k_dev, int32_t* isum_dev, int32_t* summs_dev,
                         void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ2K, "smeai_q2k_block_sums");
  if (!h) return kBadArgument;
  return q2k_block_sums(h->w, x_q8k_dev, isum_dev, summs_dev, as_stream(stream));
}

int smeai_q2k_quantize_device(const float* x_dev, int64_t n, void* y_q2k_dev, void* stream) {
  if (!x_dev || !y_q2k_dev) {
    set_last_error("smeai_q2k_quantize_device: NULL pointer");
    return kBadArgument;
  }
  return q2k_quantize(x_dev, n, y_q2k_dev, as_stream(stream));
}

int smeai_q2k_dequantize_device(const void* w_q2k_dev, int64_t n, float* y_dev, void* stream) {
  if (!w_q2k_dev || !y_dev) {
    set_last_error("smeai_q2k_dequantize_device: NULL pointer");
    return kBadArgument;
  }
  return q2k_dequantize(w_q2k_dev, n, y_dev, as_stream(stream));
}

// ---- Q3_K ----------------------------------------------------------------------

int smeai_q3k_repack(const void* w_q3k, int64_t n_rows, int64_t k, void** w_dev_out) {
  if (!w_q3k || !w_dev_out || n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("smeai_q3k_repack: bad arguments");
    return kBadArgument;
  }
  *w_dev_out = nullptr;
  if (!device_ready()) {
    set_last_error("smeai_q3k_repack: no compute-capability-10.x device");
    return kUnsupported;
  }
  Staged src;
  const size_t bytes = (size_t)n_rows * (size_t)(k / QK_K) * kQ3KBytes;
  int st = src.in(w_q3k, bytes, nullptr);
  if (st) return st;
  Handle* h = new Handle();
  st = q3k_repack(src.dev, n_rows, k, &h->w, nullptr);
  if (st == kOk && cudaStreamSynchronize(nullptr) != cudaSuccess) {
    set_last_error("smeai_q3k_repack: %s", cudaGetErrorString(cudaGetLastError()));
    st = kCudaError;
  }
  if (st) {
    if (h->w.tiles) cudaFree(h->w.tiles);
    delete h;
    return st;
  }
  *w_dev_out = h;
  return kOk;
}

void smeai_q3k_free(void* w_dev) { smeai_q2k_free(w_dev); }

int smeai_q3k_mul_mat(const void* w_dev, const void* x_q8k_dev, int64_t n_cols, float* y_dev, size_t ldy,
                      void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ3K, "smeai_q3k_mul_mat");
  if (!h) return kBadArgument;
  return q2k_gemv(h->w, x_q8k_dev, n_cols, y_dev, (int64_t)ldy, kEpiStore, nullptr, 0, as_stream(stream));
}

int smeai_q3k_mul_mat_f32(const void* w_dev, const float* x_dev, size_t ld_x, int64_t n_cols, float* y_dev,
                          size_t ldy, float rms_eps, void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ3K, "smeai_q3k_mul_mat_f32");
  if (!h) return kBadArgument;
  return q2k_gemv_any(h->w, rms_eps >= 0.f ? kInF32Rms : kInF32, x_dev, (int64_t)ld_x, rms_eps, n_cols, y_dev,
                      (int64_t)ldy, kEpiStore, nullptr, 0, as_stream(stream));
}

int smeai_q3k_block_sums(const void* w_dev, const void* x_q8k_dev, int32_t* isum_dev, int32_t* summs_dev,
                         void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ3K, "smeai_q3k_block_sums");
  if (!h) return kBadArgument;
  return q2k_block_sums(h->w, x_q8k_dev, isum_dev, summs_dev, as_stream(stream));
}

int smeai_q3k_dequantize_device(const void* w_q3k_dev, int64_t n, float* y_dev, void* stream) {
  if (!w_q3k_dev || !y_dev) {
    set_last_error("smeai_q3k_dequantize_device: NULL pointer");
    return kBadArgument;
  }
  return q3k_dequantize(w_q3k_dev, n, y_dev, as_stream(stream));
}

void dequantize_row_q3_K(const void* x, float* y, int64_t k) {
  if (!x || !y || k <= 0 || k % QK_K) {
    set_last_error("dequantize_row_q3_K: k must be a positive multiple of 256");
    return;
  }
  ThreadCtx& c = tctx();
  if (c.init() || c.a.in(x, (size_t)(k / QK_K) * kQ3KBytes, c.stream) || c.b.out(y, (size_t)k * 4) ||
      q3k_dequantize(c.a.dev, k, static_cast<float*>(c.b.dev), c.stream) || c.b.finish(c.stream) ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    if (!is_device_pointer(y)) memset(y, 0, (size_t)k * 4);
  }
}

void ggml_vec_dot_q3_K_q8_K(int n, float* s, size_t bs, const void* vx, size_t bx, const void* vy, size_t by,
                            int nrc) {
  (void)bs;
  (void)bx;
  (void)by;
  if (!s) return;
  *s = 0.f;
  if (!vx || !vy || n <= 0 || n % QK_K || nrc != 1) {
    set_last_error("ggml_vec_dot_q3_K_q8_K: needs n %% 256 == 0 and nrc == 1");
    return;
  }
  ThreadCtx& c = tctx();
  const int64_t nb = n / QK_K;
  Q2KWeight w;
  if (c.init() || c.a.in(vx, nb * kQ3KBytes, c.stream) || c.b.in(vy, nb * Q8K_BLOCK_BYTES, c.stream) ||
      c.tiles.reserve(q3k_tile_bytes(1, n)) || c.y.reserve(4) ||
      q3k_repack_into(c.a.dev, 1, n, static_cast<uint8_t*>(c.tiles.ptr), &w, c.stream) ||
      q2k_gemv(w, c.b.dev, 1, static_cast<float*>(c.y.ptr), 1, kEpiStore, nullptr, 0, c.stream) ||
      cudaMemcpyAsync(s, c.y.ptr, 4, cudaMemcpyDeviceToHost, c.stream) != cudaSuccess ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    *s = 0.f;
  }
}

// ---- Q6_K ----------------------------------------------------------------------

int smeai_q6k_repack(const void* w_q6k, int64_t n_rows, int64_t k, void** w_dev_out) {
  if (!w_q6k || !w_dev_out || n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("smeai_q6k_repack: bad arguments");
    return kBadArgument;
  }
  *w_dev_out = nullptr;
  if (!device_ready()) {
    set_last_error("smeai_q6k_repack: no compute-capability-10.x device");
    return kUnsupported;
  }
  Staged src;
  const size_t bytes = (size_t)n_rows * (size_t)(k / QK_K) * kQ6KBytes;
  int st = src.in(w_q6k, bytes, nullptr);
  if (st) return st;
  Handle* h = new Handle();
  st = q6k_repack(src.dev, n_rows, k, &h->w, nullptr);
  if (st == kOk && cudaStreamSynchronize(nullptr) != cudaSuccess) {
    set_last_error("smeai_q6k_repack: %s", cudaGetErrorString(cudaGetLastError()));
    st = kCudaError;
  }
  if (st) {
    if (h->w.tiles) cudaFree(h->w.tiles);
    delete h;
    return st;
  }
  *w_dev_out = h;
  return kOk;
}

void smeai_q6k_free(void* w_dev) { smeai_q2k_free(w_dev); }

int smeai_q6k_mul_mat(const void* w_dev, const void* x_q8k_dev, int64_t n_cols, float* y_dev, size_t ldy,
                      void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ6K, "smeai_q6k_mul_mat");
  if (!h) return kBadArgument;
  return q2k_gemv(h->w, x_q8k_dev, n_cols, y_dev, (int64_t)ldy, kEpiStore, nullptr, 0, as_stream(stream));
}

int smeai_q6k_mul_mat_f32(const void* w_dev, const float* x_dev, size_t ld_x, int64_t n_cols, float* y_dev,
                          size_t ldy, float rms_eps, void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ6K, "smeai_q6k_mul_mat_f32");
  if (!h) return kBadArgument;
  return q2k_gemv_any(h->w, rms_eps >= 0.f ? kInF32Rms : kInF32, x_dev, (int64_t)ld_x, rms_eps, n_cols, y_dev,
                      (int64_t)ldy, kEpiStore, nullptr, 0, as_stream(stream));
}

int smeai_q6k_block_sums(const void* w_dev, const void* x_q8k_dev, int32_t* isum_dev, int32_t* summs_dev,
                         void* stream) {
  const Handle* h = as_fmt(w_dev, kFmtQ6K, "smeai_q6k_block_sums");
  if (!h) return kBadArgument;
  return q2k_block_sums(h->w, x_q8k_dev, isum_dev, summs_dev, as_stream(stream));
}

int smeai_q6k_dequantize_device(const void* w_q6k_dev, int64_t n, float* y_dev, void* stream) {
  if (!w_q6k_dev || !y_dev) {
    set_last_error("smeai_q6k_dequantize_device: NULL pointer");
    return kBadArgument;
  }
  return q6k_dequantize(w_q6k_dev, n, y_dev, as_stream(stream));
}

void dequantize_row_q6_K(const void* x, float* y, int64_t k) {
  if (!x || !y || k <= 0 || k % QK_K) {
    set_last_error("dequantize_row_q6_K: k must be a positive multiple of 256");
    return;
  }
  ThreadCtx& c = tctx();
  if (c.init() || c.a.in(x, (size_t)(k / QK_K) * kQ6KBytes, c.stream) || c.b.out(y, (size_t)k * 4) ||
      q6k_dequantize(c.a.dev, k, static_cast<float*>(c.b.dev), c.stream) || c.b.finish(c.stream) ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    if (!is_device_pointer(y)) memset(y, 0, (size_t)k * 4);
  }
}

void ggml_vec_dot_q6_K_q8_K(int n, float* s, size_t bs, const void* vx, size_t bx, const void* vy, size_t by,
                            int nrc) {
  (void)bs;
  (void)bx;
  (void)by;
  if (!s) return;
  *s = 0.f;
  if (!vx || !vy || n <= 0 || n % QK_K || nrc != 1) {
    set_last_error("ggml_vec_dot_q6_K_q8_K: needs n %% 256 == 0 and nrc == 1");
    return;
  }
  ThreadCtx& c = tctx();
  const int64_t nb = n / QK_K;
  Q2KWeight w;
  if (c.init() || c.a.in(vx, nb * kQ6KBytes, c.stream) || c.b.in(vy, nb * Q8K_BLOCK_BYTES, c.stream) ||
      c.tiles.reserve(q6k_tile_bytes(1, n)) || c.y.reserve(4) ||
      q6k_repack_into(c.a.dev, 1, n, static_cast<uint8_t*>(c.tiles.ptr), &w, c.stream) ||
      q2k_gemv(w, c.b.dev, 1, static_cast<float*>(c.y.ptr), 1, kEpiStore, nullptr, 0, c.stream) ||
      cudaMemcpyAsync(s, c.y.ptr, 4, cudaMemcpyDeviceToHost, c.stream) != cudaSuccess ||
      cudaStreamSynchronize(c.stream) != cudaSuccess) {
    *s = 0.f;
  }
}

}  // extern "C"
