// api_sme_ai_ops.cu -- the C-ABI of include/sme_ai_ops.h.
//
// Argument checks run in the reference's order (args, then workspace
// capacity, then backend: sme_ai_ops.c:182-190, 434-462, 361-388) and return
// the same status codes.  Host pointers are staged through device buffers
// owned by the workspace (or, for the workspace-less *_ref_* functions, by
// the calling thread); device pointers are used in place.
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "elementwise.h"
#include "linear.h"
#include "runtime.h"
#include "../../include/sme_ai_ops.h"

using namespace smeai;

namespace {

constexpr uint32_t kWsMagic = 0x57535031u;  // "WSP1"
constexpr uint32_t kPkMagic = 0x504b5731u;  // "PKW1"

uint64_t round16(uint64_t v) { return (v + 15) / 16 * 16; }

// Library state hung off ws->a_pairs.
struct WsPriv {
  uint32_t magic = kWsMagic;
  cudaStream_t stream = nullptr;
  Staged in, out, b0, b1, b2, b3;
  DeviceBuffer raw;
  DeviceBuffer scores;  // self-attention score matrix (tiled path)  // raw weight of the "simple" path
};

// Library state behind packed->packed_weight.
struct PackedPriv {
  uint32_t magic = kPkMagic;
  int is_f32 = 0;
  void* dev = nullptr;  // [k_pad][n_pad] fp16 or fp32, zero padded
  int64_t ldb = 0;
};

WsPriv* priv(const sme_ai_workspace* ws) {
  WsPriv* p = ws ? reinterpret_cast<WsPriv*>(ws->a_pairs) : nullptr;
  return (p && p->magic == kWsMagic) ? p : nullptr;
}

const PackedPriv* ppriv(const sme_ai_packed_linear_weight* w) {
  const PackedPriv* p = w ? reinterpret_cast<const PackedPriv*>(w->packed_weight) : nullptr;
  return (p && p->magic == kPkMagic) ? p : nullptr;
}

// A CUDA failure has no reference status code; it reports UNSUPPORTED (the
// backend could not run the operator) and smeai_last_error() has the text.
sme_ai_status st(int s) { return static_cast<sme_ai_status>(s == kCudaError ? kUnsupported : s); }

// check_workspace (sme_ai_ops.c:182-190)
sme_ai_status check_ws(const sme_ai_workspace* ws, uint64_t batch, uint64_t in, uint64_t out) {
  if (!ws || !batch || !in || !out) return SME_AI_BAD_ARGUMENT;
  if (batch > ws->max_batch || in > ws->max_in_features || out > ws->max_out_features)
    return SME_AI_WORKSPACE_TOO_SMALL;
  return SME_AI_OK;
}

// Per-thread context of the workspace-less functions.
struct RefCtx {
  cudaStream_t stream = nullptr;
  Staged in, w, w2, w3, w4, out, b0, b1, b2, b3;
  DeviceBuffer t0, t1, h16;
  bool init() {
    if (!stream && cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return true;
  }
};
RefCtx& rctx() {
  thread_local RefCtx c;
  return c;
}

int sync(cudaStream_t s) {
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_last_error("%s", cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

// Packed linear on device pointers; act applied in the epilogue.
int packed_linear_dev(const __half* x, uint64_t batch, const sme_ai_packed_linear_weight* pw, const float* bias,
                      int act, float* y, cudaStream_t s) {
  const PackedPriv* p = ppriv(pw);
  return linear_f16(x, (int64_t)batch, (int64_t)pw->in_features, static_cast<const __half*>(p->dev), p->ldb,
                    (int64_t)pw->out_features, bias, act, y, s);
}

// sme_ai_linear_sme_packed_f16f32 with an activation (sme_ai_ops.c:707-729,
// 483-497): checks, staging, one fused kernel, copy back.
sme_ai_status linear_packed_act(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                const sme_ai_packed_linear_weight* pw, const float* bias, float* output, int act) {
  if (!pw || !pw->packed_weight) return SME_AI_BAD_ARGUMENT;
  sme_ai_status c = check_ws(ws, batch, pw->in_features, pw->out_features);
  if (c != SME_AI_OK) return c;
  if (!input || !output) return SME_AI_BAD_ARGUMENT;
  WsPriv* w = priv(ws);
  const PackedPriv* p = ppriv(pw);
  if (!w || !p || p->is_f32) return SME_AI_BAD_ARGUMENT;
  cudaStream_t s = w->stream;
  const uint64_t M = batch, K = pw->in_features, N = pw->out_features;
  int r = w->in.in(input, M * K * 2, s);
  if (!r) r = w->b0.in(bias, N * 4, s);
  if (!r) r = w->out.out(output, M * N * 4);
  if (!r) r = packed_linear_dev(static_cast<const __half*>(w->in.dev), M, pw, static_cast<const float*>(w->b0.dev),
                                act, static_cast<float*>(w->out.dev), s);
  if (!r) r = w->out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

// Two-layer MLP (sme_ai_ops.c:532-557): fc1 + bias + act + fp16 round in one
// kernel writing ws->tmp_f16, then fc2 + bias.
sme_ai_status mlp_packed(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                         const sme_ai_packed_linear_weight* fc1, const float* b1,
                         const sme_ai_packed_linear_weight* fc2, const float* b2, float* output, int act) {
  if (!ws || !input || !fc1 || !fc2 || !output) return SME_AI_BAD_ARGUMENT;
  if (batch > ws->max_batch || fc1->out_features > ws->max_out_features ||
      fc2->out_features > ws->max_out_features)
    return SME_AI_WORKSPACE_TOO_SMALL;
  if (!fc1->packed_weight || !fc2->packed_weight) return SME_AI_BAD_ARGUMENT;
  sme_ai_status c = check_ws(ws, batch, fc1->in_features, fc1->out_features);
  if (c != SME_AI_OK) return c;
  c = check_ws(ws, batch, fc2->in_features, fc2->out_features);
  if (c != SME_AI_OK) return c;
  if (fc1->out_features != fc2->in_features) return SME_AI_BAD_ARGUMENT;
  WsPriv* w = priv(ws);
  const PackedPriv *p1 = ppriv(fc1), *p2 = ppriv(fc2);
  if (!w || !p1 || !p2 || p1->is_f32 || p2->is_f32) return SME_AI_BAD_ARGUMENT;
  cudaStream_t s = w->stream;
  const uint64_t M = batch, K = fc1->in_features, H = fc1->out_features, N = fc2->out_features;
  __half* hid = reinterpret_cast<__half*>(ws->tmp_f16);
  int r = w->in.in(input, M * K * 2, s);
  if (!r) r = w->b0.in(b1, H * 4, s);
  if (!r) r = w->b1.in(b2, N * 4, s);
  if (!r) r = w->out.out(output, M * N * 4);
  if (!r) r = linear_f16_to_f16(static_cast<const __half*>(w->in.dev), M, K, static_cast<const __half*>(p1->dev),
                                p1->ldb, H, static_cast<const float*>(w->b0.dev), act, hid, s);
  if (!r) r = linear_f16(hid, M, H, static_cast<const __half*>(p2->dev), p2->ldb, N,
                         static_cast<const float*>(w->b1.dev), kActNone, static_cast<float*>(w->out.dev), s);
  if (!r) r = w->out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

// Reference-form Linear on the GPU: one thread per output, k ascending.
sme_ai_status linear_ref(const sme_ai_fp16* input, uint64_t batch, uint64_t in, const sme_ai_fp16* weight,
                         uint64_t out, const float* bias, float* output, int act) {
  if (!input || !weight || !output || !batch || !in || !out) return SME_AI_BAD_ARGUMENT;
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  RefCtx& c = rctx();
  if (!c.init()) return SME_AI_UNSUPPORTED;
  cudaStream_t s = c.stream;
  int r = c.in.in(input, batch * in * 2, s);
  if (!r) r = c.w.in(weight, in * out * 2, s);
  if (!r) r = c.b0.in(bias, out * 4, s);
  if (!r) r = c.out.out(output, batch * out * 4);
  if (!r) r = linear_ref_f16(static_cast<const __half*>(c.in.dev), batch, in, static_cast<const __half*>(c.w.dev),
                             out, static_cast<const float*>(c.b0.dev), act, static_cast<float*>(c.out.dev), s);
  if (!r) r = c.out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

// mlp_activation_ref / sme_ai_swiglu_ref_f16f32 on the GPU, step by step like
// the reference (sme_ai_ops.c:504-529, 1188-1225).
sme_ai_status mlp_ref(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch, uint64_t in,
                      const sme_ai_fp16* w1, uint64_t hidden, const float* b1, const sme_ai_fp16* w2, uint64_t out,
                      const float* b2, float* output, int act) {
  if (!ws || !input || !w1 || !w2 || !output) return SME_AI_BAD_ARGUMENT;
  if (batch > ws->max_batch || hidden > ws->max_out_features || out > ws->max_out_features)
    return SME_AI_WORKSPACE_TOO_SMALL;
  if (!batch || !in || !hidden || !out) return SME_AI_BAD_ARGUMENT;
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  RefCtx& c = rctx();
  if (!c.init()) return SME_AI_UNSUPPORTED;
  cudaStream_t s = c.stream;
  int r = c.in.in(input, batch * in * 2, s);
  if (!r) r = c.w.in(w1, in * hidden * 2, s);
  if (!r) r = c.w2.in(w2, hidden * out * 2, s);
  if (!r) r = c.b0.in(b1, hidden * 4, s);
  if (!r) r = c.b1.in(b2, out * 4, s);
  if (!r) r = c.out.out(output, batch * out * 4);
  if (!r) r = c.t0.reserve(batch * hidden * 4);
  if (!r) r = c.h16.reserve(batch * hidden * 2);
  float* h = static_cast<float*>(c.t0.ptr);
  __half* h16 = static_cast<__half*>(c.h16.ptr);
  if (!r) r = linear_ref_f16(static_cast<const __half*>(c.in.dev), batch, in, static_cast<const __half*>(c.w.dev),
                             hidden, static_cast<const float*>(c.b0.dev), act, h, s);
  if (!r) r = f32_to_f16(h, h16, batch * hidden, s);
  if (!r) r = linear_ref_f16(h16, batch, hidden, static_cast<const __half*>(c.w2.dev), out,
                             static_cast<const float*>(c.b1.dev), kActNone, static_cast<float*>(c.out.dev), s);
  if (!r) r = c.out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

// Elementwise helpers: a per-thread context, synchronous, silent on errors.
struct EwCtx {
  cudaStream_t stream = nullptr;
  Staged a, b, o;
  bool init() {
    if (!stream && cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return true;
  }
};
EwCtx& ectx() {
  thread_local EwCtx c;
  return c;
}

template <typename F>
void ew_binary(float* output, const float* lhs, const float* rhs, uint64_t count, F f) {
  if (!output || !lhs || !rhs || !count) return;
  EwCtx& c = ectx();
  if (!c.init()) return;
  int r = c.a.in(lhs, count * 4, c.stream);
  if (!r) r = c.b.in(rhs, count * 4, c.stream);
  if (!r) r = c.o.out(output, count * 4);
  if (!r) r = f(static_cast<float*>(c.o.dev), static_cast<const float*>(c.a.dev),
                static_cast<const float*>(c.b.dev), (int64_t)count, c.stream);
  if (!r) r = c.o.finish(c.stream);
  if (!r) sync(c.stream);
}

void ew_act(float* data, uint64_t count, int act) {
  if (!data || !count) return;
  EwCtx& c = ectx();
  if (!c.init()) return;
  int r = c.a.in(data, count * 4, c.stream);
  if (!r) {
    // in place: the staged copy is the output
    c.o.dev = c.a.dev;
    c.o.host = (c.a.dev == data) ? nullptr : data;
    c.o.n = count * 4;
    r = act_inplace(static_cast<float*>(c.a.dev), (int64_t)count, act, c.stream);
  }
  if (!r) r = c.o.finish(c.stream);
  if (!r) sync(c.stream);
  c.o.host = nullptr;
}

// ---- fixed scratch for sme_ai_swiglu_packed_f16f32_noalloc ------------------
// The fp16 hidden state of that entry point lives in this file-scope device
// array, not in a workspace, so the entry point never allocates.  Its size is
// fixed: batch * hidden_features must not exceed kNoAllocHiddenElems
// (524288 fp16 values = 1 MiB).  Every GPU that loads the library holds the
// array until the process exits.  In host code `g_noalloc_hidden` is only a
// stand-in symbol, not a device address: the address is fetched once per
// device with cudaGetSymbolAddress and passed to the kernels.  The cached
// address is never looked up again, so it is valid only while the context it
// came from lives (a cudaDeviceReset loads the module anew; the public header
// says the entry point must not be used on a device reset after its first call).
constexpr uint64_t kNoAllocHiddenElems = 512u * 1024u;
static __device__ __align__(256) __half g_noalloc_hidden[kNoAllocHiddenElems];

std::mutex g_noalloc_mu;
__half* g_noalloc_ptr[64] = {nullptr};

// Device address of the scratch on the current device (set up on first use).
int noalloc_scratch(__half** out) {
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_last_error("device ordinal %d out of range", dev);
    return kUnsupported;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_hidden);
    if (e != cudaSuccess || !p) {
      set_last_error("cudaGetSymbolAddress of the fixed scratch failed: %s", cudaGetErrorString(e));
      return kCudaError;
    }
    g_noalloc_ptr[dev] = static_cast<__half*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return kOk;
}

}  // namespace

extern "C" {

int sme_ai_has_sme(void) { return device_ready() ? 1 : 0; }
int sme_ai_has_sme2(void) { return 0; }
uint64_t sme_ai_cntb(void) { return 64; }
uint64_t sme_ai_cntw(void) { return 16; }

sme_ai_status sme_ai_workspace_init(sme_ai_workspace* ws, uint64_t max_batch, uint64_t max_in_features,
                                    uint64_t max_out_features) {
  if (!ws || !max_batch || !max_in_features || !max_out_features) return SME_AI_BAD_ARGUMENT;
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  memset(ws, 0, sizeof(*ws));
  ws->cntb = 64;
  ws->cntw = 16;
  ws->max_batch = max_batch;
  ws->max_in_features = max_in_features;
  ws->max_out_features = max_out_features;
  ws->max_h = max_in_features;
  ws->max_m_pad = round16(max_batch);
  ws->max_k_pad = round16(max_in_features);
  ws->max_n_pad = round16(max_out_features);
  WsPriv* p = new WsPriv();
  ws->a_pairs = reinterpret_cast<float*>(p);
  const uint64_t hid = max_batch * max_out_features;
  bool ok = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking) == cudaSuccess;
  ok = ok && device_malloc((void**)&ws->tmp_f32, hid * 4) == cudaSuccess;
  ok = ok && device_malloc((void**)&ws->tmp2_f32, hid * 4) == cudaSuccess;
  ok = ok && device_malloc((void**)&ws->tmp_f16, hid * 2) == cudaSuccess;
  ok = ok && device_malloc((void**)&ws->b_pack, ws->max_k_pad * ws->max_n_pad * 2) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    sme_ai_workspace_destroy(ws);
    return SME_AI_ALLOC_FAILED;
  }
  return SME_AI_OK;
}

void sme_ai_workspace_destroy(sme_ai_workspace* ws) {
  if (!ws) return;
  WsPriv* p = priv(ws);
  if (p) {
    if (p->stream) {
      cudaStreamSynchronize(p->stream);
      cudaStreamDestroy(p->stream);
    }
    p->magic = 0;
    delete p;
  }
  if (ws->tmp_f32) cudaFree(ws->tmp_f32);
  if (ws->tmp2_f32) cudaFree(ws->tmp2_f32);
  if (ws->tmp_f16) cudaFree(ws->tmp_f16);
  if (ws->b_pack) cudaFree(ws->b_pack);
  memset(ws, 0, sizeof(*ws));
}

static sme_ai_status packed_init(sme_ai_packed_linear_weight* packed, const void* weight, uint64_t in,
                                 uint64_t out, bool f32) {
  if (!packed || !weight || !in || !out) return SME_AI_BAD_ARGUMENT;
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  memset(packed, 0, sizeof(*packed));
  packed->k_pad = round16(in);
  packed->n_pad = round16(out);
  PackedPriv* p = new PackedPriv();
  p->is_f32 = f32 ? 1 : 0;
  p->ldb = (int64_t)packed->n_pad;
  const size_t esz = f32 ? 4 : 2;
  if (device_malloc((void**)&p->dev, packed->k_pad * packed->n_pad * esz) != cudaSuccess) {
    cudaGetLastError();
    delete p;
    return SME_AI_ALLOC_FAILED;
  }
  // Copy the raw [in][out] weight row by row into the padded layout.
  cudaError_t e = cudaMemset(p->dev, 0, packed->k_pad * packed->n_pad * esz);
  if (e == cudaSuccess)
    e = cudaMemcpy2D(p->dev, packed->n_pad * esz, weight, out * esz, out * esz, in, cudaMemcpyDefault);
  if (e != cudaSuccess) {
    set_last_error("packed weight upload: %s", cudaGetErrorString(e));
    cudaFree(p->dev);
    delete p;
    return SME_AI_ALLOC_FAILED;
  }
  packed->in_features = in;
  packed->out_features = out;
  packed->packed_weight = reinterpret_cast<float*>(p);
  return SME_AI_OK;
}

sme_ai_status sme_ai_packed_linear_weight_init(sme_ai_packed_linear_weight* packed, const sme_ai_fp16* weight,
                                               uint64_t in_features, uint64_t out_features) {
  return packed_init(packed, weight, in_features, out_features, false);
}

sme_ai_status sme_ai_packed_linear_weight_init_f32(sme_ai_packed_linear_weight* packed, const float* weight,
                                                   uint64_t in_features, uint64_t out_features) {
  return packed_init(packed, weight, in_features, out_features, true);
}

void sme_ai_packed_linear_weight_destroy(sme_ai_packed_linear_weight* packed) {
  if (!packed) return;
  PackedPriv* p = const_cast<PackedPriv*>(ppriv(packed));
  if (p) {
    if (p->dev) cudaFree(p->dev);
    p->magic = 0;
    delete p;
  }
  memset(packed, 0, sizeof(*packed));
}

// ---- Linear ------------------------------------------------------------------
sme_ai_status sme_ai_linear_ref_f16f32(const sme_ai_fp16* input, uint64_t batch, uint64_t in_features,
                                       const sme_ai_fp16* weight, uint64_t out_features, const float* bias,
                                       float* output) {
  return linear_ref(input, batch, in_features, weight, out_features, bias, output, kActNone);
}

sme_ai_status sme_ai_linear_sme_simple_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                              uint64_t in_features, const sme_ai_fp16* weight,
                                              uint64_t out_features, const float* bias, float* output) {
  sme_ai_status c = check_ws(ws, batch, in_features, out_features);
  if (c != SME_AI_OK) return c;
  if (!weight || !input || !output) return SME_AI_BAD_ARGUMENT;
  WsPriv* w = priv(ws);
  if (!w) return SME_AI_BAD_ARGUMENT;
  // Pack the raw weight into ws->b_pack on every call (the reference repacks
  // into ws->b_pack the same way, sme_ai_ops.c:673-705).
  cudaStream_t s = w->stream;
  const uint64_t kp = round16(in_features), np = round16(out_features);
  __half* bp = reinterpret_cast<__half*>(ws->b_pack);
  Staged raw;
  int r = raw.in(weight, in_features * out_features * 2, s);
  if (!r) r = pack_weight_f16(static_cast<const __half*>(raw.dev), in_features, out_features, bp, kp, np, s);
  if (!r) r = w->in.in(input, batch * in_features * 2, s);
  if (!r) r = w->b0.in(bias, out_features * 4, s);
  if (!r) r = w->out.out(output, batch * out_features * 4);
  if (!r) r = linear_f16(static_cast<const __half*>(w->in.dev), batch, in_features, bp, np, out_features,
                         static_cast<const float*>(w->b0.dev), kActNone, static_cast<float*>(w->out.dev), s);
  if (!r) r = w->out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

sme_ai_status sme_ai_linear_sme_packed_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                              const sme_ai_packed_linear_weight* packed_weight, const float* bias,
                                              float* output) {
  return linear_packed_act(ws, input, batch, packed_weight, bias, output, kActNone);
}

sme_ai_status sme_ai_linear_relu_ref_f16f32(const sme_ai_fp16* input, uint64_t batch, uint64_t in_features,
                                            const sme_ai_fp16* weight, uint64_t out_features, const float* bias,
                                            float* output) {
  return linear_ref(input, batch, in_features, weight, out_features, bias, output, kActRelu);
}
sme_ai_status sme_ai_linear_relu_sme_packed_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input,
                                                   uint64_t batch, const sme_ai_packed_linear_weight* pw,
                                                   const float* bias, float* output) {
  return linear_packed_act(ws, input, batch, pw, bias, output, kActRelu);
}
sme_ai_status sme_ai_linear_gelu_ref_f16f32(const sme_ai_fp16* input, uint64_t batch, uint64_t in_features,
                                            const sme_ai_fp16* weight, uint64_t out_features, const float* bias,
                                            float* output) {
  return linear_ref(input, batch, in_features, weight, out_features, bias, output, kActGelu);
}
sme_ai_status sme_ai_linear_gelu_sme_packed_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input,
                                                   uint64_t batch, const sme_ai_packed_linear_weight* pw,
                                                   const float* bias, float* output) {
  return linear_packed_act(ws, input, batch, pw, bias, output, kActGelu);
}
sme_ai_status sme_ai_linear_silu_ref_f16f32(const sme_ai_fp16* input, uint64_t batch, uint64_t in_features,
                                            const sme_ai_fp16* weight, uint64_t out_features, const float* bias,
                                            float* output) {
  return linear_ref(input, batch, in_features, weight, out_features, bias, output, kActSilu);
}
sme_ai_status sme_ai_linear_silu_sme_packed_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input,
                                                   uint64_t batch, const sme_ai_packed_linear_weight* pw,
                                                   const float* bias, float* output) {
  return linear_packed_act(ws, input, batch, pw, bias, output, kActSilu);
}

// ---- MLP -----------------------------------------------------------------------
sme_ai_status sme_ai_mlp_relu_ref_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                         uint64_t in_features, const sme_ai_fp16* fc1_weight,
                                         uint64_t hidden_features, const float* fc1_bias,
                                         const sme_ai_fp16* fc2_weight, uint64_t out_features,
                                         const float* fc2_bias, float* output) {
  return mlp_ref(ws, input, batch, in_features, fc1_weight, hidden_features, fc1_bias, fc2_weight, out_features,
                 fc2_bias, output, kActRelu);
}
sme_ai_status sme_ai_mlp_relu_sme_packed_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                                const sme_ai_packed_linear_weight* fc1, const float* b1,
                                                const sme_ai_packed_linear_weight* fc2, const float* b2,
                                                float* output) {
  return mlp_packed(ws, input, batch, fc1, b1, fc2, b2, output, kActRelu);
}
sme_ai_status sme_ai_mlp_gelu_ref_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                         uint64_t in_features, const sme_ai_fp16* fc1_weight,
                                         uint64_t hidden_features, const float* fc1_bias,
                                         const sme_ai_fp16* fc2_weight, uint64_t out_features,
                                         const float* fc2_bias, float* output) {
  return mlp_ref(ws, input, batch, in_features, fc1_weight, hidden_features, fc1_bias, fc2_weight, out_features,
                 fc2_bias, output, kActGelu);
}
sme_ai_status sme_ai_mlp_gelu_sme_packed_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                                const sme_ai_packed_linear_weight* fc1, const float* b1,
                                                const sme_ai_packed_linear_weight* fc2, const float* b2,
                                                float* output) {
  return mlp_packed(ws, input, batch, fc1, b1, fc2, b2, output, kActGelu);
}

// ---- SwiGLU --------------------------------------------------------------------
sme_ai_status sme_ai_swiglu_ref_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                       uint64_t in_features, const sme_ai_fp16* gate_weight,
                                       uint64_t hidden_features, const float* gate_bias,
                                       const sme_ai_fp16* up_weight, const float* up_bias,
                                       const sme_ai_fp16* down_weight, uint64_t out_features,
                                       const float* down_bias, float* output) {
  if (!ws || !input || !gate_weight || !up_weight || !down_weight || !output) return SME_AI_BAD_ARGUMENT;
  if (batch > ws->max_batch || hidden_features > ws->max_out_features || out_features > ws->max_out_features)
    return SME_AI_WORKSPACE_TOO_SMALL;
  if (!batch || !in_features || !hidden_features || !out_features) return SME_AI_BAD_ARGUMENT;
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  RefCtx& c = rctx();
  if (!c.init()) return SME_AI_UNSUPPORTED;
  cudaStream_t s = c.stream;
  const uint64_t M = batch, K = in_features, H = hidden_features, N = out_features;
  int r = c.in.in(input, M * K * 2, s);
  if (!r) r = c.w.in(gate_weight, K * H * 2, s);
  if (!r) r = c.w2.in(up_weight, K * H * 2, s);
  if (!r) r = c.w3.in(down_weight, H * N * 2, s);
  if (!r) r = c.b0.in(gate_bias, H * 4, s);
  if (!r) r = c.b1.in(up_bias, H * 4, s);
  if (!r) r = c.b2.in(down_bias, N * 4, s);
  if (!r) r = c.out.out(output, M * N * 4);
  if (!r) r = c.t0.reserve(M * H * 4);
  if (!r) r = c.t1.reserve(M * H * 4);
  if (!r) r = c.h16.reserve(M * H * 2);
  float *g = static_cast<float*>(c.t0.ptr), *u = static_cast<float*>(c.t1.ptr);
  __half* h16 = static_cast<__half*>(c.h16.ptr);
  const __half* x = static_cast<const __half*>(c.in.dev);
  if (!r) r = linear_ref_f16(x, M, K, static_cast<const __half*>(c.w.dev), H, static_cast<const float*>(c.b0.dev),
                             kActNone, g, s);
  if (!r) r = linear_ref_f16(x, M, K, static_cast<const __half*>(c.w2.dev), H,
                             static_cast<const float*>(c.b1.dev), kActNone, u, s);
  if (!r) r = silu_mul_f16(g, u, h16, M * H, s);
  if (!r) r = linear_ref_f16(h16, M, H, static_cast<const __half*>(c.w3.dev), N,
                             static_cast<const float*>(c.b2.dev), kActNone, static_cast<float*>(c.out.dev), s);
  if (!r) r = c.out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

sme_ai_status sme_ai_swiglu_sme_packed_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t batch,
                                              const sme_ai_packed_linear_weight* gate_weight,
                                              const float* gate_bias,
                                              const sme_ai_packed_linear_weight* up_weight, const float* up_bias,
                                              const sme_ai_packed_linear_weight* down_weight,
                                              const float* down_bias, float* output) {
  if (!ws || !input || !gate_weight || !up_weight || !down_weight || !output) return SME_AI_BAD_ARGUMENT;
  if (batch > ws->max_batch || gate_weight->out_features > ws->max_out_features ||
      up_weight->out_features > ws->max_out_features || down_weight->out_features > ws->max_out_features)
    return SME_AI_WORKSPACE_TOO_SMALL;
  if (gate_weight->out_features != up_weight->out_features ||
      gate_weight->out_features != down_weight->in_features)
    return SME_AI_BAD_ARGUMENT;
  if (gate_weight->in_features != up_weight->in_features) return SME_AI_BAD_ARGUMENT;
  if (!gate_weight->packed_weight || !up_weight->packed_weight || !down_weight->packed_weight)
    return SME_AI_BAD_ARGUMENT;
  sme_ai_status c = check_ws(ws, batch, gate_weight->in_features, gate_weight->out_features);
  if (c != SME_AI_OK) return c;
  c = check_ws(ws, batch, down_weight->in_features, down_weight->out_features);
  if (c != SME_AI_OK) return c;
  WsPriv* w = priv(ws);
  const PackedPriv *pg = ppriv(gate_weight), *pu = ppriv(up_weight), *pd = ppriv(down_weight);
  if (!w || !pg || !pu || !pd || pg->is_f32 || pu->is_f32 || pd->is_f32) return SME_AI_BAD_ARGUMENT;
  cudaStream_t s = w->stream;
  const uint64_t M = batch, K = gate_weight->in_features, H = gate_weight->out_features,
                 N = down_weight->out_features;
  __half* hid = reinterpret_cast<__half*>(ws->tmp_f16);
  int r = w->in.in(input, M * K * 2, s);
  if (!r) r = w->b0.in(gate_bias, H * 4, s);
  if (!r) r = w->b1.in(up_bias, H * 4, s);
  if (!r) r = w->b2.in(down_bias, N * 4, s);
  if (!r) r = w->out.out(output, M * N * 4);
  if (!r) r = swiglu_gate_up_f16(static_cast<const __half*>(w->in.dev), M, K, static_cast<const __half*>(pg->dev),
                                 static_cast<const __half*>(pu->dev), pg->ldb, H,
                                 static_cast<const float*>(w->b0.dev), static_cast<const float*>(w->b1.dev), hid, s);
  if (!r) r = linear_f16(hid, M, H, static_cast<const __half*>(pd->dev), pd->ldb, N,
                         static_cast<const float*>(w->b2.dev), kActNone, static_cast<float*>(w->out.dev), s);
  if (!r) r = w->out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

// ---- self-attention (sme_ai_ops.c:1320-1499) -------------------------------------
// Shared argument checks of both variants (:1343-1350 / :1435-1442).
static sme_ai_status attention_checks(const sme_ai_workspace* ws, const void* input, uint64_t seq_len,
                                      uint64_t model_dim, uint64_t num_heads, const void* q, const void* k,
                                      const void* v, const void* o, const float* output) {
  if (!ws || !input || !q || !k || !v || !o || !output || !seq_len || !model_dim || !num_heads ||
      model_dim % num_heads)
    return SME_AI_BAD_ARGUMENT;
  if (seq_len > ws->max_batch || model_dim > ws->max_in_features || model_dim > ws->max_out_features)
    return SME_AI_WORKSPACE_TOO_SMALL;
  return SME_AI_OK;
}

// Q -> ws->tmp_f32, K -> ws->tmp2_f32 and V -> the output buffer, as the
// reference places them; the attention kernel writes the fp16 context to
// ws->tmp_f16 and the output projection overwrites V.
sme_ai_status sme_ai_self_attention_ref_f16f32(sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t seq_len,
                                               uint64_t model_dim, uint64_t num_heads, const sme_ai_fp16* q_weight,
                                               const float* q_bias, const sme_ai_fp16* k_weight, const float* k_bias,
                                               const sme_ai_fp16* v_weight, const float* v_bias,
                                               const sme_ai_fp16* out_weight, const float* out_bias, int causal,
                                               float* output) {
  sme_ai_status c =
      attention_checks(ws, input, seq_len, model_dim, num_heads, q_weight, k_weight, v_weight, out_weight, output);
  if (c != SME_AI_OK) return c;
  if (!priv(ws)) return SME_AI_BAD_ARGUMENT;
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  RefCtx& x = rctx();
  if (!x.init()) return SME_AI_UNSUPPORTED;
  cudaStream_t s = x.stream;
  const uint64_t S = seq_len, D = model_dim;
  float *q = ws->tmp_f32, *k = ws->tmp2_f32;
  __half* ctx16 = reinterpret_cast<__half*>(ws->tmp_f16);
  int r = x.in.in(input, S * D * 2, s);
  if (!r) r = x.w.in(q_weight, D * D * 2, s);
  if (!r) r = x.w2.in(k_weight, D * D * 2, s);
  if (!r) r = x.w3.in(v_weight, D * D * 2, s);
  if (!r) r = x.w4.in(out_weight, D * D * 2, s);
  if (!r) r = x.b0.in(q_bias, D * 4, s);
  if (!r) r = x.b1.in(k_bias, D * 4, s);
  if (!r) r = x.b2.in(v_bias, D * 4, s);
  if (!r) r = x.b3.in(out_bias, D * 4, s);
  if (!r) r = x.out.out(output, S * D * 4);
  const __half* in = static_cast<const __half*>(x.in.dev);
  float* v = static_cast<float*>(x.out.dev);
  if (!r) r = linear_ref_f16(in, S, D, static_cast<const __half*>(x.w.dev), D, static_cast<const float*>(x.b0.dev),
                             kActNone, q, s);
  if (!r) r = linear_ref_f16(in, S, D, static_cast<const __half*>(x.w2.dev), D, static_cast<const float*>(x.b1.dev),
                             kActNone, k, s);
  if (!r) r = linear_ref_f16(in, S, D, static_cast<const __half*>(x.w3.dev), D, static_cast<const float*>(x.b2.dev),
                             kActNone, v, s);
  DeviceBuffer& sc = priv(ws)->scores;
  const size_t sc_bytes = attention_scratch_bytes(S, D, num_heads);
  if (!r && sc_bytes) r = sc.reserve(sc_bytes);
  if (!r) r = attention_core(q, k, v, S, D, num_heads, causal, ctx16, static_cast<float*>(sc.ptr), sc.cap, s);
  if (!r) r = linear_ref_f16(ctx16, S, D, static_cast<const __half*>(x.w4.dev), D,
                             static_cast<const float*>(x.b3.dev), kActNone, v, s);
  if (!r) r = x.out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

// Checks of the packed variant beyond the shared ones (:1443-1448).
static sme_ai_status attention_packed_checks(uint64_t model_dim, const sme_ai_packed_linear_weight* const (&pw)[4],
                                             const PackedPriv* (&pp)[4]) {
  for (int t = 0; t < 4; ++t) {
    if (pw[t]->in_features != model_dim || pw[t]->out_features != model_dim) return SME_AI_BAD_ARGUMENT;
    pp[t] = ppriv(pw[t]);
    if (!pp[t] || pp[t]->is_f32) return SME_AI_BAD_ARGUMENT;
  }
  return SME_AI_OK;
}

// The packed attention on device pointers, queued on s: projections into
// ws->tmp_f32 (Q), ws->tmp2_f32 (K) and `out` (V), the attention kernel into
// ws->tmp_f16, the output projection over V.
static int attention_packed_dev(sme_ai_workspace* ws, const __half* in, uint64_t S, uint64_t D, uint64_t heads,
                                const sme_ai_packed_linear_weight* const (&pw)[4], const float* const (&bias)[4],
                                int causal, float* out, cudaStream_t s) {
  float *q = ws->tmp_f32, *k = ws->tmp2_f32;
  __half* ctx16 = reinterpret_cast<__half*>(ws->tmp_f16);
  int r = packed_linear_dev(in, S, pw[0], bias[0], kActNone, q, s);
  if (!r) r = packed_linear_dev(in, S, pw[1], bias[1], kActNone, k, s);
  if (!r) r = packed_linear_dev(in, S, pw[2], bias[2], kActNone, out, s);
  DeviceBuffer& sc = priv(ws)->scores;
  const size_t sc_bytes = attention_scratch_bytes(S, D, heads);
  if (!r && sc_bytes) r = sc.reserve(sc_bytes);
  if (!r) r = attention_core(q, k, out, S, D, heads, causal, ctx16, static_cast<float*>(sc.ptr), sc.cap, s);
  if (!r) r = packed_linear_dev(ctx16, S, pw[3], bias[3], kActNone, out, s);
  return r;
}

sme_ai_status sme_ai_self_attention_sme_packed_f16f32(
    sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t seq_len, uint64_t model_dim, uint64_t num_heads,
    const sme_ai_packed_linear_weight* q_weight, const float* q_bias, const sme_ai_packed_linear_weight* k_weight,
    const float* k_bias, const sme_ai_packed_linear_weight* v_weight, const float* v_bias,
    const sme_ai_packed_linear_weight* out_weight, const float* out_bias, int causal, float* output) {
  sme_ai_status c =
      attention_checks(ws, input, seq_len, model_dim, num_heads, q_weight, k_weight, v_weight, out_weight, output);
  if (c != SME_AI_OK) return c;
  const sme_ai_packed_linear_weight* const pw[4] = {q_weight, k_weight, v_weight, out_weight};
  const PackedPriv* pp[4];
  c = attention_packed_checks(model_dim, pw, pp);
  if (c != SME_AI_OK) return c;
  WsPriv* w = priv(ws);
  if (!w) return SME_AI_BAD_ARGUMENT;
  cudaStream_t s = w->stream;
  const uint64_t S = seq_len, D = model_dim;
  int r = w->in.in(input, S * D * 2, s);
  if (!r) r = w->b0.in(q_bias, D * 4, s);
  if (!r) r = w->b1.in(k_bias, D * 4, s);
  if (!r) r = w->b2.in(v_bias, D * 4, s);
  if (!r) r = w->b3.in(out_bias, D * 4, s);
  if (!r) r = w->out.out(output, S * D * 4);
  const float* const bias[4] = {static_cast<const float*>(w->b0.dev), static_cast<const float*>(w->b1.dev),
                                static_cast<const float*>(w->b2.dev), static_cast<const float*>(w->b3.dev)};
  if (!r) r = attention_packed_dev(ws, static_cast<const __half*>(w->in.dev), S, D, num_heads, pw, bias, causal,
                                   static_cast<float*>(w->out.dev), s);
  if (!r) r = w->out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

sme_ai_status sme_ai_self_attention_packed_f16f32_device(
    sme_ai_workspace* ws, const sme_ai_fp16* input, uint64_t seq_len, uint64_t model_dim, uint64_t num_heads,
    const sme_ai_packed_linear_weight* q_weight, const float* q_bias, const sme_ai_packed_linear_weight* k_weight,
    const float* k_bias, const sme_ai_packed_linear_weight* v_weight, const float* v_bias,
    const sme_ai_packed_linear_weight* out_weight, const float* out_bias, int causal, float* output, void* stream) {
  sme_ai_status c =
      attention_checks(ws, input, seq_len, model_dim, num_heads, q_weight, k_weight, v_weight, out_weight, output);
  if (c != SME_AI_OK) return c;
  const sme_ai_packed_linear_weight* const pw[4] = {q_weight, k_weight, v_weight, out_weight};
  const PackedPriv* pp[4];
  c = attention_packed_checks(model_dim, pw, pp);
  if (c != SME_AI_OK) return c;
  if (!priv(ws)) return SME_AI_BAD_ARGUMENT;
  const float* const bias[4] = {q_bias, k_bias, v_bias, out_bias};
  return st(attention_packed_dev(ws, reinterpret_cast<const __half*>(input), seq_len, model_dim, num_heads, pw, bias,
                                 causal, output, static_cast<cudaStream_t>(stream)));
}

sme_ai_status sme_ai_self_attention_core_f32_device(const float* q, const float* k, const float* v, uint64_t seq_len,
                                                    uint64_t model_dim, uint64_t num_heads, int causal,
                                                    sme_ai_fp16* context, void* stream) {
  if (!q || !k || !v || !context || !seq_len || !model_dim || !num_heads || model_dim % num_heads)
    return SME_AI_BAD_ARGUMENT;
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  thread_local DeviceBuffer sc;
  const size_t sc_bytes = attention_scratch_bytes((int64_t)seq_len, (int64_t)model_dim, (int64_t)num_heads);
  if (sc_bytes) {
    const int r = sc.reserve(sc_bytes);
    if (r) return st(r);
  }
  return st(attention_core(q, k, v, (int64_t)seq_len, (int64_t)model_dim, (int64_t)num_heads, causal,
                           reinterpret_cast<__half*>(context), static_cast<float*>(sc.ptr), sc.cap,
                           static_cast<cudaStream_t>(stream)));
}

// ---- elementwise -----------------------------------------------------------------
void sme_ai_add_f32(float* output, const float* lhs, const float* rhs, uint64_t count) {
  ew_binary(output, lhs, rhs, count, ew_add);
}
void sme_ai_mul_f32(float* output, const float* lhs, const float* rhs, uint64_t count) {
  ew_binary(output, lhs, rhs, count, ew_mul);
}
void sme_ai_residual_add_f32(float* output, const float* input, const float* residual, uint64_t count) {
  ew_binary(output, input, residual, count, ew_add);
}
void sme_ai_add_bias_rowwise_f32(float* output, const float* input, const float* bias, uint64_t rows,
                                 uint64_t cols) {
  if (!output || !input || !rows || !cols) return;
  EwCtx& c = ectx();
  if (!c.init()) return;
  int r = c.a.in(input, rows * cols * 4, c.stream);
  if (!r) r = c.b.in(bias, cols * 4, c.stream);
  if (!r) r = c.o.out(output, rows * cols * 4);
  if (!r) r = ew_bias_rows(static_cast<float*>(c.o.dev), static_cast<const float*>(c.a.dev),
                           static_cast<const float*>(c.b.dev), (int64_t)rows, (int64_t)cols, c.stream);
  if (!r) r = c.o.finish(c.stream);
  if (!r) sync(c.stream);
}
void sme_ai_relu_inplace_f32(float* data, uint64_t count) { ew_act(data, count, kActRelu); }
void sme_ai_gelu_inplace_f32(float* data, uint64_t count) { ew_act(data, count, kActGelu); }
void sme_ai_silu_inplace_f32(float* data, uint64_t count) { ew_act(data, count, kActSilu); }

// ---- additions -----------------------------------------------------------------------
sme_ai_status sme_ai_linear_sme_packed_f32f32(sme_ai_workspace* ws, const float* input, uint64_t batch,
                                              const sme_ai_packed_linear_weight* pw, const float* bias,
                                              float* output) {
  if (!pw || !pw->packed_weight) return SME_AI_BAD_ARGUMENT;
  sme_ai_status c = check_ws(ws, batch, pw->in_features, pw->out_features);
  if (c != SME_AI_OK) return c;
  if (!input || !output) return SME_AI_BAD_ARGUMENT;
  WsPriv* w = priv(ws);
  const PackedPriv* p = ppriv(pw);
  if (!w || !p || !p->is_f32) return SME_AI_BAD_ARGUMENT;
  cudaStream_t s = w->stream;
  const uint64_t M = batch, K = pw->in_features, N = pw->out_features;
  int r = w->in.in(input, M * K * 4, s);
  if (!r) r = w->b0.in(bias, N * 4, s);
  if (!r) r = w->out.out(output, M * N * 4);
  if (!r) r = linear_f32(static_cast<const float*>(w->in.dev), M, K, static_cast<const float*>(p->dev), p->ldb, N,
                         static_cast<const float*>(w->b0.dev), kActNone, static_cast<float*>(w->out.dev), s);
  if (!r) r = w->out.finish(s);
  if (!r) r = sync(s);
  return st(r);
}

sme_ai_status sme_ai_linear_packed_f16f32_device(const sme_ai_fp16* input, uint64_t batch,
                                                 const sme_ai_packed_linear_weight* pw, const float* bias, int act,
                                                 float* output, void* stream) {
  if (!pw || !pw->packed_weight || !input || !output || !batch) return SME_AI_BAD_ARGUMENT;
  const PackedPriv* p = ppriv(pw);
  if (!p || p->is_f32 || act < kActNone || act > kActSilu) return SME_AI_BAD_ARGUMENT;
  return st(packed_linear_dev(reinterpret_cast<const __half*>(input), batch, pw, bias, act, output,
                              static_cast<cudaStream_t>(stream)));
}


// SwiGLU on packed weights that allocates nothing (see sme_ai_ops.h).  Same
// kernels and same results as sme_ai_swiglu_sme_packed_f16f32; the hidden
// state goes to the fixed device array above instead of ws->tmp_f16.
sme_ai_status sme_ai_swiglu_packed_f16f32_noalloc(const sme_ai_fp16* input, uint64_t batch,
                                                  const sme_ai_packed_linear_weight* gate_weight,
                                                  const float* gate_bias,
                                                  const sme_ai_packed_linear_weight* up_weight, const float* up_bias,
                                                  const sme_ai_packed_linear_weight* down_weight,
                                                  const float* down_bias, float* output, void* stream) {
  if (!input || !gate_weight || !up_weight || !down_weight || !output || !batch) return SME_AI_BAD_ARGUMENT;
  if (!gate_weight->packed_weight || !up_weight->packed_weight || !down_weight->packed_weight)
    return SME_AI_BAD_ARGUMENT;
  if (gate_weight->out_features != up_weight->out_features ||
      gate_weight->out_features != down_weight->in_features || gate_weight->in_features != up_weight->in_features)
    return SME_AI_BAD_ARGUMENT;
  const PackedPriv *pg = ppriv(gate_weight), *pu = ppriv(up_weight), *pd = ppriv(down_weight);
  if (!pg || !pu || !pd || pg->is_f32 || pu->is_f32 || pd->is_f32) return SME_AI_BAD_ARGUMENT;
  const uint64_t M = batch, K = gate_weight->in_features, H = gate_weight->out_features,
                 N = down_weight->out_features;
  if (H > kNoAllocHiddenElems || M > kNoAllocHiddenElems / H) {
    set_last_error("sme_ai_swiglu_packed_f16f32_noalloc: batch*hidden_features = %llu exceeds the fixed "
                   "scratch of %llu fp16 values",
                   (unsigned long long)(M * H), (unsigned long long)kNoAllocHiddenElems);
    return SME_AI_WORKSPACE_TOO_SMALL;
  }
  if (!device_ready()) return SME_AI_UNSUPPORTED;
  __half* hid = nullptr;
  int r = noalloc_scratch(&hid);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!r) r = swiglu_gate_up_f16(reinterpret_cast<const __half*>(input), M, K, static_cast<const __half*>(pg->dev),
                                 static_cast<const __half*>(pu->dev), pg->ldb, H, gate_bias, up_bias, hid, s);
  if (!r) r = linear_f16(hid, M, H, static_cast<const __half*>(pd->dev), pd->ldb, N, down_bias, kActNone, output, s);
  return st(r);
}

}  // extern "C"
