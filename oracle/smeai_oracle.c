/*
 * smeai_oracle.c -- CPU restatement of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests, the smoke check and the CPU
 * baseline leg of the benchmark, never by the product library.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  Contraction is
 * disabled so that every fused multiply-add below is an explicit fmaf() and the
 * float semantics are stated in the source, not chosen by the compiler.
 */
#include "smeai_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32.  _Float16 is IEEE binary16, the same storage as the       */
/* reference's __fp16 (sme_ai_library/include/sme_ai_ops.h:75); conversions  */
/* to half round to nearest-even, conversions to float are exact.            */
/* ------------------------------------------------------------------------ */
float orc_half_to_float(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float) v;
}

uint16_t orc_float_to_half(float f) {
    _Float16 v = (_Float16) f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

void orc_halves_to_floats(const uint16_t *src, float *dst, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = orc_half_to_float(src[i]);
}

void orc_floats_to_halves(const float *src, uint16_t *dst, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = orc_float_to_half(src[i]);
}

/* ------------------------------------------------------------------------ */
/* The reference benches' deterministic data: a 32-bit LCG                   */
/* (state = state*1664525 + 1013904223), value (r % 2001)/2000 - 0.5,        */
/* rounded to fp16 for half inputs.                                           */
/* sme_ai_library/test_bench/bench_sme_full_timing.c:33-51                    */
/* sme_ai_library/test_bench/verify_sme_ai_timing.c:68-86                     */
/* ------------------------------------------------------------------------ */
static float lcg_value(uint32_t *state) {
    *state = *state * 1664525u + 1013904223u;
    return ((float) (*state % 2001u) / 2000.0f) - 0.5f;
}

void orc_lcg_fill_f16(uint16_t *dst, uint64_t count, uint32_t seed) {
    uint32_t s = seed;
    for (uint64_t i = 0; i < count; ++i) dst[i] = orc_float_to_half(lcg_value(&s));
}

void orc_lcg_fill_f32(float *dst, uint64_t count, uint32_t seed) {
    uint32_t s = seed;
    for (uint64_t i = 0; i < count; ++i) dst[i] = lcg_value(&s);
}

/* ======================================================================== */
/* Path A: sme_ai_library                                                    */
/* ======================================================================== */

/* gelu_approx, sme_ai_ops.c:107-112 (tanh form, libm tanhf). */
static float gelu_tanh(float x) {
    const float c0 = 0.7978845608f;
    const float c1 = 0.044715f;
    float cube = x * x * x;
    float inner = c0 * (x + c1 * cube);
    return 0.5f * x * (1.0f + tanhf(inner));
}

/* Activations applied in place after the GEMM + bias.
 * ReLU: sme_ai_ops.c:834-846 (max(x, 0)); GELU: :867-874 via gelu_approx;
 * SiLU: :879-887 (x / (1 + expf(-x))). */
static void apply_act(float *v, uint64_t n, int act) {
    for (uint64_t i = 0; i < n; ++i) {
        float x = v[i];
        switch (act) {
            case ORC_ACT_RELU: v[i] = x > 0.0f ? x : 0.0f; break;
            case ORC_ACT_GELU: v[i] = gelu_tanh(x); break;
            case ORC_ACT_SILU: v[i] = x / (1.0f + expf(-x)); break;
            default: break;
        }
    }
}

/* Row-wise bias add after the GEMM; a NULL bias is allowed.
 * add_bias_f32, sme_ai_ops.c:207-221. */
static void add_bias(float *out, const float *bias, uint64_t rows, uint64_t cols) {
    if (bias == NULL) return;
    for (uint64_t r = 0; r < rows; ++r)
        for (uint64_t c = 0; c < cols; ++c) out[r * cols + c] += bias[c];
}

/*
 * Linear on fp16 data: out[r][c] = sum_k in[r][k] * w[k][c], k ascending, in
 * fp32, then + bias, then the activation.
 *   scalar_matmul_f16f16_f32   sme_ai_ops.c:251-267
 *   sme_ai_linear_ref_f16f32   sme_ai_ops.c:653-671
 *   linear_activation_ref      sme_ai_ops.c:465-480
 * The product of two fp16 values is exact in fp32, so the fused form below is
 * bit-identical to the reference's unfused acc += a*b under any contraction.
 */
int orc_linear_f16f32(const uint16_t *input, uint64_t batch, uint64_t in_features,
                      const uint16_t *weight, uint64_t out_features,
                      const float *bias, float *output, int act) {
    if (!input || !weight || !output || !batch || !in_features || !out_features) return -1;
    float *wf = (float *) malloc(in_features * out_features * sizeof(float));
    float *xf = (float *) malloc(batch * in_features * sizeof(float));
    if (!wf || !xf) { free(wf); free(xf); return -2; }
    orc_halves_to_floats(weight, wf, in_features * out_features);
    orc_halves_to_floats(input, xf, batch * in_features);
    for (uint64_t r = 0; r < batch; ++r) {
        for (uint64_t c = 0; c < out_features; ++c) {
            float acc = 0.0f;
            for (uint64_t k = 0; k < in_features; ++k)
                acc = fmaf(xf[r * in_features + k], wf[k * out_features + c], acc);
            output[r * out_features + c] = acc;
        }
    }
    free(wf);
    free(xf);
    add_bias(output, bias, batch, out_features);
    apply_act(output, batch * out_features, act);
    return 0;
}

/*
 * The same operator for true fp32 inputs (a new-API variant with no reference
 * counterpart; it keeps scalar_matmul_f16f16_f32's loop order).  The multiply
 * -add is fused, which is what the reference's GCC build (default
 * -ffp-contract=fast on an FMA target) makes of acc += a*b.
 */
int orc_linear_f32f32(const float *input, uint64_t batch, uint64_t in_features,
                      const float *weight, uint64_t out_features,
                      const float *bias, float *output, int act) {
    if (!input || !weight || !output || !batch || !in_features || !out_features) return -1;
    for (uint64_t r = 0; r < batch; ++r) {
        for (uint64_t c = 0; c < out_features; ++c) {
            float acc = 0.0f;
            for (uint64_t k = 0; k < in_features; ++k)
                acc = fmaf(input[r * in_features + k], weight[k * out_features + c], acc);
            output[r * out_features + c] = acc;
        }
    }
    add_bias(output, bias, batch, out_features);
    apply_act(output, batch * out_features, act);
    return 0;
}

/*
 * Two-layer MLP: h = act(in*W1 + b1) rounded to fp16, out = h*W2 + b2.
 * mlp_activation_ref, sme_ai_ops.c:504-529 (fp16 re-round via
 * convert_fp32_to_fp16, :175-179).
 */
int orc_mlp_f16f32(const uint16_t *input, uint64_t batch, uint64_t in_features,
                   const uint16_t *fc1_weight, uint64_t hidden_features, const float *fc1_bias,
                   const uint16_t *fc2_weight, uint64_t out_features, const float *fc2_bias,
                   float *output, int act) {
    float *h = (float *) malloc(batch * hidden_features * sizeof(float));
    uint16_t *h16 = (uint16_t *) malloc(batch * hidden_features * sizeof(uint16_t));
    int rc = -2;
    if (h && h16) {
        rc = orc_linear_f16f32(input, batch, in_features, fc1_weight, hidden_features, fc1_bias, h, act);
        if (rc == 0) {
            orc_floats_to_halves(h, h16, batch * hidden_features);
            rc = orc_linear_f16f32(h16, batch, hidden_features, fc2_weight, out_features, fc2_bias,
                                   output, ORC_ACT_NONE);
        }
    }
    free(h);
    free(h16);
    return rc;
}

/*
 * SwiGLU: g = in*Wg + bg, u = in*Wu + bu, h = fp16(silu(g) * u),
 * out = h*Wd + bd.   sme_ai_swiglu_ref_f16f32, sme_ai_ops.c:1188-1225
 * (silu :879-887, elementwise mul :801-814, fp16 round :175-179).
 */
int orc_swiglu_f16f32(const uint16_t *input, uint64_t batch, uint64_t in_features,
                      const uint16_t *gate_weight, uint64_t hidden_features, const float *gate_bias,
                      const uint16_t *up_weight, const float *up_bias,
                      const uint16_t *down_weight, uint64_t out_features, const float *down_bias,
                      float *output) {
    uint64_t n = batch * hidden_features;
    float *g = (float *) malloc(n * sizeof(float));
    float *u = (float *) malloc(n * sizeof(float));
    uint16_t *h16 = (uint16_t *) malloc(n * sizeof(uint16_t));
    int rc = -2;
    if (g && u && h16) {
        rc = orc_linear_f16f32(input, batch, in_features, gate_weight, hidden_features, gate_bias, g, ORC_ACT_NONE);
        if (rc == 0)
            rc = orc_linear_f16f32(input, batch, in_features, up_weight, hidden_features, up_bias, u, ORC_ACT_NONE);
        if (rc == 0) {
            for (uint64_t i = 0; i < n; ++i) {
                float s = g[i] / (1.0f + expf(-g[i]));
                h16[i] = orc_float_to_half(s * u[i]);
            }
            rc = orc_linear_f16f32(h16, batch, hidden_features, down_weight, out_features, down_bias,
                                   output, ORC_ACT_NONE);
        }
    }
    free(g);
    free(u);
    free(h16);
    return rc;
}

/*
 * dot_f32_sve, sme_ai_ops.c:1268-1279: 16 float lanes (the 512-bit vector the
 * API reports), lane l accumulating elements l, l+16, ... with a fused
 * multiply-add (svmla); svaddv then reduces the lanes.  svaddv's order is
 * implementation-defined; this restatement reduces pairwise (lane l + lane
 * l+8, then +4, +2, +1), the order the device kernel uses.
 */
static float attn_dot(const float *a, const float *b, uint64_t n) {
    float acc[16];
    for (int l = 0; l < 16; ++l) acc[l] = 0.0f;
    for (uint64_t i = 0; i < n; ++i) acc[i & 15] = fmaf(a[i], b[i], acc[i & 15]);
    for (int w = 8; w >= 1; w >>= 1)
        for (int l = 0; l < w; ++l) acc[l] = acc[l] + acc[l + w];
    return acc[0];
}

/*
 * Softmax of one score row in place: max, e_j = expf(v_j - max) summed
 * sequentially (j ascending), then e_j / sum; a zero sum gives zeros.
 * Causal rows replace v_j (j > i) by -1e30.
 *   sme_ai_softmax_masked_rowwise_f32   sme_ai_ops.c:893-933
 *   sme_ai_softmax_causal_rowwise_f32   sme_ai_ops.c:935-973
 */
static void attn_softmax_row(float *row, uint64_t n, uint64_t i, int causal) {
    float mx = -INFINITY, sum = 0.0f;
    for (uint64_t j = 0; j < n; ++j) {
        float v = (causal && j > i) ? -1.0e30f : row[j];
        if (v > mx) mx = v;
    }
    for (uint64_t j = 0; j < n; ++j) {
        float v = (causal && j > i) ? -1.0e30f : row[j];
        float ex = expf(v - mx);
        row[j] = ex;
        sum += ex;
    }
    for (uint64_t j = 0; j < n; ++j) row[j] = (sum == 0.0f) ? 0.0f : row[j] / sum;
}

/*
 * Self-attention, sme_ai_self_attention_ref_f16f32 (sme_ai_ops.c:1320-1410):
 *   Q, K, V = Linear(input) (k-ascending fp32 sums, + bias)
 *   per head h (columns h*hd .. h*hd+hd-1, hd = model_dim / num_heads):
 *     s_ij = dot(Q_i, K_j) * (1 / sqrtf(hd))      (attn_dot)
 *     p_i  = softmax(s_i)                          (causal or not)
 *     ctx_i = sum_j p_ij * V_j, j ascending, ctx = ctx + v*p unfused
 *       (attention_weighted_sum_f32, :1287-1318: svmul_n then svadd)
 *   output = Linear(fp16(ctx), out_weight) + out_bias.
 * The reference writes V into `output` first and reuses one score buffer per
 * head; neither changes a value.
 */
int orc_self_attention_f16f32(const uint16_t *input, uint64_t seq_len, uint64_t model_dim, uint64_t num_heads,
                              const uint16_t *q_weight, const float *q_bias,
                              const uint16_t *k_weight, const float *k_bias,
                              const uint16_t *v_weight, const float *v_bias,
                              const uint16_t *out_weight, const float *out_bias,
                              int causal, float *output, uint16_t *context16) {
    if (!input || !q_weight || !k_weight || !v_weight || !out_weight || !output || !seq_len || !model_dim ||
        !num_heads || model_dim % num_heads)
        return -1;
    const uint64_t S = seq_len, D = model_dim, hd = model_dim / num_heads;
    const float scale = 1.0f / sqrtf((float) hd);
    float *q = (float *) malloc(S * D * sizeof(float));
    float *k = (float *) malloc(S * D * sizeof(float));
    float *v = (float *) malloc(S * D * sizeof(float));
    float *ctx = (float *) malloc(S * D * sizeof(float));
    float *sc = (float *) malloc(S * S * sizeof(float));
    uint16_t *c16 = (uint16_t *) malloc(S * D * sizeof(uint16_t));
    int rc = -2;
    if (q && k && v && ctx && sc && c16) {
        rc = orc_linear_f16f32(input, S, D, q_weight, D, q_bias, q, ORC_ACT_NONE);
        if (!rc) rc = orc_linear_f16f32(input, S, D, k_weight, D, k_bias, k, ORC_ACT_NONE);
        if (!rc) rc = orc_linear_f16f32(input, S, D, v_weight, D, v_bias, v, ORC_ACT_NONE);
        for (uint64_t h = 0; !rc && h < num_heads; ++h) {
            const uint64_t off = h * hd;
            for (uint64_t i = 0; i < S; ++i)
                for (uint64_t j = 0; j < S; ++j) sc[i * S + j] = attn_dot(q + i * D + off, k + j * D + off, hd) * scale;
            for (uint64_t i = 0; i < S; ++i) attn_softmax_row(sc + i * S, S, i, causal);
            for (uint64_t i = 0; i < S; ++i) {
                float *c = ctx + i * D + off;
                for (uint64_t d = 0; d < hd; ++d) c[d] = 0.0f;
                for (uint64_t j = 0; j < S; ++j) {
                    const float p = sc[i * S + j];
                    const float *vr = v + j * D + off;
                    for (uint64_t d = 0; d < hd; ++d) {
                        float t = vr[d] * p;
                        c[d] = c[d] + t;
                    }
                }
            }
        }
        if (!rc) {
            orc_floats_to_halves(ctx, c16, S * D);
            if (context16) memcpy(context16, c16, S * D * sizeof(uint16_t));
            rc = orc_linear_f16f32(c16, S, D, out_weight, D, out_bias, output, ORC_ACT_NONE);
        }
    }
    free(q);
    free(k);
    free(v);
    free(ctx);
    free(sc);
    free(c16);
    return rc;
}

/*
 * The reference's packed layout: packed[n_tile][k_pad][16] fp32, zero padded,
 * k_pad/n_pad = round_up(., 16).  prepack_weight_fp16_to_sme_tiles,
 * sme_ai_ops.c:281-301.  (Used by tests to document the reference layout.)
 */
void orc_pack_weight_f16_tiles(const uint16_t *weight, float *packed,
                               uint64_t in_features, uint64_t out_features) {
    uint64_t kpad = (in_features + 15) / 16 * 16;
    uint64_t npad = (out_features + 15) / 16 * 16;
    memset(packed, 0, kpad * npad * sizeof(float));
    for (uint64_t c = 0; c < out_features; ++c)
        for (uint64_t k = 0; k < in_features; ++k)
            packed[(c / 16) * kpad * 16 + k * 16 + (c % 16)] =
                orc_half_to_float(weight[k * out_features + c]);
}

/* ======================================================================== */
/* Path B: ggml Q2_K x Q8_K (ggml 0.9.8 generic C, restated)                 */
/* ======================================================================== */

/*
 * ggml's nearest_int: add 1.5*2^23 so that the float adder rounds to an
 * integer (round-half-to-even), then read the integer out of the mantissa.
 * Valid for |v| < 2^22.
 */
static int magic_round(float v_plus_magic) {
    int32_t bits;
    memcpy(&bits, &v_plus_magic, 4);
    return (bits & 0x007fffff) - 0x00400000;
}
static const float kMagic = 12582912.0f;

static int round_separate(float v) { return magic_round(v + kMagic); }

/*
 * quantize_row_q8_K (ggml-quants.c quantize_row_q8_K_ref; the activation
 * quantizer the reference's Q2_K path runs on every src1 row,
 * llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:127-131).  Per 256 values:
 *   - pick the value of largest magnitude (first one on ties), call it max;
 *   - an all-zero block gives d = 0 and zero quants (bsums written as 0);
 *   - iscale = -127/max; q = nearest(iscale*x) capped at 127;
 *   - bsums[j] = sum of q[16j .. 16j+15];  d = 1/iscale.
 * rounding = ORC_Q8K_ROUND_FUSED evaluates nearest(iscale*x) as one fused
 * multiply-add with the magic constant -- what GCC's default
 * -ffp-contract=fast makes of the inlined nearest_int on an FMA target such
 * as the reference's AArch64 build; ORC_Q8K_ROUND_SEPARATE rounds the product
 * first (a -ffp-contract=off build).
 */
void orc_quantize_row_q8_K(const float *x, orc_block_q8_K *y, int64_t k, int rounding) {
    int64_t nb = k / ORC_QK_K;
    for (int64_t b = 0; b < nb; ++b) {
        const float *xb = x + b * ORC_QK_K;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < ORC_QK_K; ++j) {
            float a = fabsf(xb[j]);
            if (a > amax) { amax = a; vmax = xb[j]; }
        }
        memset(y[b].bsums, 0, sizeof(y[b].bsums));
        if (amax == 0.0f) {
            y[b].d = 0.0f;
            memset(y[b].qs, 0, sizeof(y[b].qs));
            continue;
        }
        float iscale = -127.0f / vmax;
        for (int j = 0; j < ORC_QK_K; ++j) {
            int q = rounding == ORC_Q8K_ROUND_FUSED ? magic_round(fmaf(iscale, xb[j], kMagic))
                                                    : round_separate(iscale * xb[j]);
            y[b].qs[j] = (int8_t) (q > 127 ? 127 : q);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += y[b].qs[16 * g + i];
            y[b].bsums[g] = (int16_t) s;
        }
        y[b].d = 1.0f / iscale;
    }
}

/*
 * make_qkx2_quants restated (ggml-quants.c): fit x ~ scale*L + min over one
 * 16-value group with L in [0, nmax], weighted by w, starting from the
 * (min, max) range and then trying nstep+1 perturbed inverse scales with a
 * weighted least-squares (scale, min) refit, keeping the best mean-absolute
 * error.  Returns the scale; *neg_min receives -min (>= 0).
 */
static float fit_group(int n, int nmax, const float *x, const float *w, uint8_t *L,
                       float *neg_min, float rmin, float rdelta, int nstep) {
    uint8_t trial[16];
    float lo = x[0], hi = x[0];
    float sw = w[0], swx = w[0] * x[0];
    for (int i = 1; i < n; ++i) {
        if (x[i] < lo) lo = x[i];
        if (x[i] > hi) hi = x[i];
        sw += w[i];
        swx += w[i] * x[i];
    }
    if (lo > 0.0f) lo = 0.0f;
    if (hi == lo) {
        memset(L, 0, (size_t) n);
        *neg_min = -lo;
        return 0.0f;
    }
    float inv = (float) nmax / (hi - lo);
    float scale = 1.0f / inv;
    float best = 0.0f;
    for (int i = 0; i < n; ++i) {
        int l = round_separate(inv * (x[i] - lo));
        l = l < 0 ? 0 : (l > nmax ? nmax : l);
        L[i] = (uint8_t) l;
        float diff = scale * (float) l + lo - x[i];
        best += w[i] * fabsf(diff);
    }
    for (int step = 0; step <= nstep; ++step) {
        float inv_t = (rmin + rdelta * (float) step + (float) nmax) / (hi - lo);
        float sl = 0.0f, sl2 = 0.0f, sxl = 0.0f;
        for (int i = 0; i < n; ++i) {
            int l = round_separate(inv_t * (x[i] - lo));
            l = l < 0 ? 0 : (l > nmax ? nmax : l);
            trial[i] = (uint8_t) l;
            sl += w[i] * (float) l;
            sl2 += w[i] * (float) l * (float) l;
            sxl += w[i] * (float) l * x[i];
        }
        float det = sw * sl2 - sl * sl;
        if (det > 0.0f) {
            float s_t = (sw * sxl - swx * sl) / det;
            float m_t = (sl2 * swx - sl * sxl) / det;
            if (m_t > 0.0f) {
                m_t = 0.0f;
                s_t = sxl / sl2;
            }
            float err = 0.0f;
            for (int i = 0; i < n; ++i) {
                float diff = s_t * (float) trial[i] + m_t - x[i];
                err += w[i] * fabsf(diff);
            }
            if (err < best) {
                memcpy(L, trial, (size_t) n);
                best = err;
                scale = s_t;
                lo = m_t;
            }
        }
    }
    *neg_min = -lo;
    return scale;
}

/*
 * quantize_row_q2_K (ggml-quants.c quantize_row_q2_K_ref restated): per
 * 16-value group fit (scale, min) with fit_group(nmax = 3, rmin = -0.5,
 * rdelta = 0.1, nstep = 15, |x| weights); quantize the 16 scales and 16 mins
 * to 4 bits against their maxima (d = max_scale/15, dmin = max_min/15, fp16);
 * requantize every value against the 4-bit-rounded (scale, min); pack four
 * 2-bit values per byte, byte l of each 32-byte half holding values
 * l, l+32, l+64, l+96 of that 128-value half at bit offsets 0, 2, 4, 6.
 * This is the weight generator for tests and benchmarks; parity of the
 * hot path is defined on identical blocks, so bit-identity with ggml's own
 * quantizer is not required (and is not claimed).
 */
void orc_quantize_row_q2_K(const float *x, orc_block_q2_K *y, int64_t k) {
    int64_t nb = k / ORC_QK_K;
    for (int64_t b = 0; b < nb; ++b) {
        const float *xb = x + b * ORC_QK_K;
        uint8_t L[ORC_QK_K];
        float wts[16], scales[16], mins[16];
        float max_scale = 0.0f, max_min = 0.0f;
        for (int g = 0; g < 16; ++g) {
            for (int i = 0; i < 16; ++i) wts[i] = fabsf(xb[16 * g + i]);
            scales[g] = fit_group(16, 3, xb + 16 * g, wts, L + 16 * g, &mins[g], -0.5f, 0.1f, 15);
            if (scales[g] > max_scale) max_scale = scales[g];
            if (mins[g] > max_min) max_min = mins[g];
        }
        memset(y[b].scales, 0, 16);
        if (max_scale > 0.0f) {
            float inv = 15.0f / max_scale;
            for (int g = 0; g < 16; ++g) y[b].scales[g] = (uint8_t) round_separate(inv * scales[g]);
            y[b].d = orc_float_to_half(max_scale / 15.0f);
        } else {
            y[b].d = orc_float_to_half(0.0f);
        }
        if (max_min > 0.0f) {
            float inv = 15.0f / max_min;
            for (int g = 0; g < 16; ++g)
                y[b].scales[g] |= (uint8_t) (round_separate(inv * mins[g]) << 4);
            y[b].dmin = orc_float_to_half(max_min / 15.0f);
        } else {
            y[b].dmin = orc_float_to_half(0.0f);
        }
        float dd = orc_half_to_float(y[b].d), dm = orc_half_to_float(y[b].dmin);
        for (int g = 0; g < 16; ++g) {
            float ds = dd * (float) (y[b].scales[g] & 0xF);
            if (ds == 0.0f) continue;
            float ms = dm * (float) (y[b].scales[g] >> 4);
            for (int i = 0; i < 16; ++i) {
                int l = round_separate((xb[16 * g + i] + ms) / ds);
                L[16 * g + i] = (uint8_t) (l < 0 ? 0 : (l > 3 ? 3 : l));
            }
        }
        for (int half = 0; half < 2; ++half)
            for (int l = 0; l < 32; ++l) {
                const uint8_t *s = L + half * 128 + l;
                y[b].qs[half * 32 + l] = (uint8_t) (s[0] | (s[32] << 2) | (s[64] << 4) | (s[96] << 6));
            }
    }
}

/* Value i of a Q2_K block: d*sc_j*q_i - dmin*m_j, j = i/16 (the layout
 * gguf-py Q2_K.dequantize_blocks decodes, gguf/quants.py:404-428). */
void orc_dequantize_row_q2_K(const orc_block_q2_K *x, float *y, int64_t k) {
    int64_t nb = k / ORC_QK_K;
    for (int64_t b = 0; b < nb; ++b) {
        float d = orc_half_to_float(x[b].d), dmin = orc_half_to_float(x[b].dmin);
        for (int i = 0; i < ORC_QK_K; ++i) {
            int half = i / 128, within = i % 128, shift = 2 * (within / 32), l = within % 32;
            int q = (x[b].qs[half * 32 + l] >> shift) & 3;
            int j = i / 16;
            float dl = d * (float) (x[b].scales[j] & 0xF);
            float ml = dmin * (float) (x[b].scales[j] >> 4);
            y[b * ORC_QK_K + i] = dl * (float) q - ml;
        }
    }
}

/*
 * The integer part of ggml_vec_dot_q2_K_q8_K (generic C) for each super-block:
 *   isum  = sum_j sc_j * sum_{i in sub-block j} q2_i * q8_i
 *   summs = sum_j m_j  * bsums_j
 * These are exact integers; the GPU kernels must reproduce them bit for bit.
 */
void orc_q2k_block_sums(int n, const orc_block_q2_K *x, const orc_block_q8_K *y,
                        int32_t *isum, int32_t *summs) {
    int nb = n / ORC_QK_K;
    for (int b = 0; b < nb; ++b) {
        const uint8_t *sc = x[b].scales;
        int32_t mm = 0;
        for (int j = 0; j < 16; ++j) mm += (int32_t) y[b].bsums[j] * (int32_t) (sc[j] >> 4);
        /* ggml's generic loop nest: two 128-value halves, four 2-bit planes per
         * half, each plane two 16-value sub-blocks with their own scale. */
        const uint8_t *q2 = x[b].qs;
        const int8_t *q8 = y[b].qs;
        int32_t acc = 0;
        int j = 0;
        for (int half = 0; half < 2; ++half) {
            for (int shift = 0; shift < 8; shift += 2) {
                int32_t lo = 0, hi = 0;
                for (int l = 0; l < 16; ++l) lo += (int32_t) q8[l] * ((q2[l] >> shift) & 3);
                for (int l = 16; l < 32; ++l) hi += (int32_t) q8[l] * ((q2[l] >> shift) & 3);
                acc += (int32_t) (sc[j] & 0xF) * lo;
                acc += (int32_t) (sc[j + 1] & 0xF) * hi;
                j += 2;
                q8 += 32;
            }
            q2 += 32;
        }
        isum[b] = acc;
        summs[b] = mm;
    }
}

/*
 * ggml_vec_dot_q2_K_q8_K (generic C, nrc == 1): per super-block
 *   dall = d_y * fp32(d_x),  dmin = d_y * fp32(dmin_x)
 *   sumf += dall*isum - dmin*summs          (blocks in ascending order)
 * combine = ORC_COMBINE_FUSED evaluates the term as
 * fmaf(dall, isum, -(dmin*summs)), which is what GCC's default contraction
 * forms from that expression on an FMA target (the first product is fused
 * into the subtraction); ORC_COMBINE_SEPARATE rounds both products.
 */
float orc_vec_dot_q2_K_q8_K(int n, const orc_block_q2_K *x, const orc_block_q8_K *y, int combine) {
    int nb = n / ORC_QK_K;
    float sumf = 0.0f;
    for (int b = 0; b < nb; ++b) {
        int32_t isum, summs;
        orc_q2k_block_sums(ORC_QK_K, x + b, y + b, &isum, &summs);
        float dall = y[b].d * orc_half_to_float(x[b].d);
        float dmin = y[b].d * orc_half_to_float(x[b].dmin);
        float term;
        if (combine == ORC_COMBINE_FUSED) {
            term = fmaf(dall, (float) isum, -(dmin * (float) summs));
        } else {
            float t1 = dall * (float) isum;
            float t2 = dmin * (float) summs;
            term = t1 - t2;
        }
        sumf = sumf + term;
    }
    return sumf;
}

/*
 * mul_mat of a Q2_K weight [n_rows, k] with Q8_K activations [n_cols, k]:
 * y[c*ldy + r] = vec_dot(row r, col c) -- ggml's dst layout (ne0 = rows
 * contiguous).  Rows are split over n_threads like ggml's CPU threads.
 */
void orc_q2k_mul_mat(const orc_block_q2_K *w, int64_t n_rows, int64_t k,
                     const orc_block_q8_K *xq, int64_t n_cols, float *y, int64_t ldy,
                     int combine, int n_threads) {
    int64_t nb = k / ORC_QK_K;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for schedule(static) num_threads(n_threads)
#endif
    for (int64_t r = 0; r < n_rows; ++r)
        for (int64_t c = 0; c < n_cols; ++c)
            y[c * ldy + r] = orc_vec_dot_q2_K_q8_K((int) k, w + r * nb, xq + c * nb, combine);
    (void) n_threads;
}

/* ======================================================================== */
/* Q3_K (ggml 0.9.8 generic C; the reference leaves its 110 Q3_K tensors on  */
/* that path, llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:44-51).  A weight is     */
/* d * (scale_j - 32) * q with q = low 2 bits - (high bit clear ? 4 : 0),    */
/* q in [-4, 3]; the 2-bit planes and sub-block order are Q2_K's, the high   */
/* bit of quant (half h, plane s, byte l) is bit 4h+s of hmask[l].           */
/* ======================================================================== */

/* The 16 scales minus 32 from the 12 packed bytes: scales 0-7 take their low
 * 4 bits from the nibbles of bytes 0-7 (low nibbles first), scales 8-15 from
 * the high nibbles; the top 2 bits come from bytes 8-11, two per scale. */
void orc_q3k_scales(const orc_block_q3_K *x, int8_t sc[16]) {
    for (int j = 0; j < 16; ++j) {
        int lo = (j < 8) ? (x->scales[j] & 0xF) : (x->scales[j - 8] >> 4);
        int hi = (x->scales[8 + (j % 4)] >> (2 * (j / 4))) & 3;
        sc[j] = (int8_t) ((lo | (hi << 4)) - 32);
    }
}

static int orc_q3k_quant(const orc_block_q3_K *x, int i) {
    int half = i / 128, within = i % 128, shift = within / 32, l = within % 32;
    int q = (x->qs[half * 32 + l] >> (2 * shift)) & 3;
    int hbit = (x->hmask[l] >> (4 * half + shift)) & 1;
    return q - (hbit ? 0 : 4);
}

void orc_dequantize_row_q3_K(const orc_block_q3_K *x, float *y, int64_t k) {
    int64_t nb = k / ORC_QK_K;
    for (int64_t b = 0; b < nb; ++b) {
        int8_t sc[16];
        orc_q3k_scales(x + b, sc);
        float d = orc_half_to_float(x[b].d);
        for (int i = 0; i < ORC_QK_K; ++i) {
            float dl = d * (float) sc[i / 16];
            y[b * ORC_QK_K + i] = dl * (float) orc_q3k_quant(x + b, i);
        }
    }
}

/* Per super-block: isum = sum_j (scale_j - 32) * sum_{i in j} q_i * q8_i. */
void orc_q3k_block_sums(int n, const orc_block_q3_K *x, const orc_block_q8_K *y, int32_t *isum) {
    int nb = n / ORC_QK_K;
    for (int b = 0; b < nb; ++b) {
        int8_t sc[16];
        orc_q3k_scales(x + b, sc);
        int32_t acc = 0;
        for (int j = 0; j < 16; ++j) {
            int32_t s = 0;
            for (int i = 16 * j; i < 16 * j + 16; ++i) s += (int32_t) y[b].qs[i] * orc_q3k_quant(x + b, i);
            acc += (int32_t) sc[j] * s;
        }
        isum[b] = acc;
    }
}

/*
 * ggml_vec_dot_q3_K_q8_K, generic C (order = ORC_Q3K_GGML): the integer
 * products go to 8 lanes by position mod 8, aux32[l] = sum over the block of
 * (scale_j - 32) * q_i * q8_i for i = l (mod 8); per block
 * d = fp32(d_x) * d_y and sums[l] += d * aux32[l] (one fused multiply-add,
 * what GCC's default contraction forms on an FMA target); the result is
 * sums[0] + sums[1] + ... + sums[7].  order = ORC_Q3K_BLOCK_ORDER: the GPU
 * kernels' combine, sumf += (fp32(d_x) * d_y) * isum per block in ascending
 * order (the same integers, one float accumulator).
 */
float orc_vec_dot_q3_K_q8_K(int n, const orc_block_q3_K *x, const orc_block_q8_K *y, int order) {
    int nb = n / ORC_QK_K;
    if (order == ORC_Q3K_BLOCK_ORDER) {
        float sumf = 0.0f;
        for (int b = 0; b < nb; ++b) {
            int32_t isum;
            orc_q3k_block_sums(ORC_QK_K, x + b, y + b, &isum);
            const float d = orc_half_to_float(x[b].d) * y[b].d;
            sumf = sumf + d * (float) isum;
        }
        return sumf;
    }
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < nb; ++b) {
        int8_t sc[16];
        orc_q3k_scales(x + b, sc);
        int32_t aux32[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 16; ++j)
            for (int i = 16 * j; i < 16 * j + 16; ++i)
                aux32[i % 8] += (int32_t) sc[j] * ((int32_t) y[b].qs[i] * orc_q3k_quant(x + b, i));
        const float d = orc_half_to_float(x[b].d) * y[b].d;
        for (int l = 0; l < 8; ++l) sums[l] = fmaf(d, (float) aux32[l], sums[l]);
    }
    float sumf = 0.0f;
    for (int l = 0; l < 8; ++l) sumf += sums[l];
    return sumf;
}

void orc_q3k_mul_mat(const orc_block_q3_K *w, int64_t n_rows, int64_t k,
                     const orc_block_q8_K *xq, int64_t n_cols, float *y, int64_t ldy,
                     int order, int n_threads) {
    int64_t nb = k / ORC_QK_K;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for schedule(static) num_threads(n_threads)
#endif
    for (int64_t r = 0; r < n_rows; ++r)
        for (int64_t c = 0; c < n_cols; ++c)
            y[c * ldy + r] = orc_vec_dot_q3_K_q8_K((int) k, w + r * nb, xq + c * nb, order);
    (void) n_threads;
}

/* ======================================================================== */
/* Q6_K (ggml 0.9.8 generic C; the one Q6_K tensor of the reference's model,  */
/* llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:44-51).  Weight i of a 128-weight    */
/* half (l = i % 32, group g = i / 32) is d * scale_{i/16} * (u - 32) with     */
/* u = (low or high nibble of ql[l + 32*(g&1)]) | (bits 2g..2g+1 of qh[l])<<4 */
/* (low nibble for g < 2, high for g >= 2).                                  */
/* ======================================================================== */
static int orc_q6k_quant(const orc_block_q6_K *x, int i) {
    int half = i / 128, within = i % 128, g = within / 32, l = within % 32;
    const uint8_t *ql = x->ql + 64 * half, *qh = x->qh + 32 * half;
    int lo = ql[l + 32 * (g & 1)];
    lo = (g < 2) ? (lo & 0xF) : (lo >> 4);
    int hi = (qh[l] >> (2 * g)) & 3;
    return (lo | (hi << 4)) - 32;
}

void orc_dequantize_row_q6_K(const orc_block_q6_K *x, float *y, int64_t k) {
    int64_t nb = k / ORC_QK_K;
    for (int64_t b = 0; b < nb; ++b) {
        float d = orc_half_to_float(x[b].d);
        for (int i = 0; i < ORC_QK_K; ++i) {
            float dl = d * (float) x[b].scales[i / 16];
            y[b * ORC_QK_K + i] = dl * (float) orc_q6k_quant(x + b, i);
        }
    }
}

/* Per super-block: isum = sum_j scale_j * sum_{i in j} q_i * q8_i. */
void orc_q6k_block_sums(int n, const orc_block_q6_K *x, const orc_block_q8_K *y, int32_t *isum) {
    int nb = n / ORC_QK_K;
    for (int b = 0; b < nb; ++b) {
        int32_t acc = 0;
        for (int j = 0; j < 16; ++j) {
            int32_t s = 0;
            for (int i = 16 * j; i < 16 * j + 16; ++i) s += (int32_t) y[b].qs[i] * orc_q6k_quant(x + b, i);
            acc += (int32_t) x[b].scales[j] * s;
        }
        isum[b] = acc;
    }
}

/* ggml_vec_dot_q6_K_q8_K, generic C: the 8-lane form of the Q3_K dot above
 * (aux32[l] over positions i = l mod 8, sums[l] = fmaf(d, aux32[l], sums[l]),
 * then sums[0] + ... + sums[7]); ORC_Q3K_BLOCK_ORDER is the GPU's combine,
 * sumf += (fp32(d_x) * d_y) * fp32(isum) per block. */
float orc_vec_dot_q6_K_q8_K(int n, const orc_block_q6_K *x, const orc_block_q8_K *y, int order) {
    int nb = n / ORC_QK_K;
    if (order == ORC_Q3K_BLOCK_ORDER) {
        float sumf = 0.0f;
        for (int b = 0; b < nb; ++b) {
            int32_t isum;
            orc_q6k_block_sums(ORC_QK_K, x + b, y + b, &isum);
            const float d = orc_half_to_float(x[b].d) * y[b].d;
            sumf = sumf + d * (float) isum;
        }
        return sumf;
    }
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < nb; ++b) {
        int32_t aux32[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 16; ++j)
            for (int i = 16 * j; i < 16 * j + 16; ++i)
                aux32[i % 8] += (int32_t) x[b].scales[j] * ((int32_t) y[b].qs[i] * orc_q6k_quant(x + b, i));
        const float d = orc_half_to_float(x[b].d) * y[b].d;
        for (int l = 0; l < 8; ++l) sums[l] = fmaf(d, (float) aux32[l], sums[l]);
    }
    float sumf = 0.0f;
    for (int l = 0; l < 8; ++l) sumf += sums[l];
    return sumf;
}

void orc_q6k_mul_mat(const orc_block_q6_K *w, int64_t n_rows, int64_t k,
                     const orc_block_q8_K *xq, int64_t n_cols, float *y, int64_t ldy,
                     int order, int n_threads) {
    int64_t nb = k / ORC_QK_K;
#ifdef _OPENMP
    if (n_threads < 1) n_threads = 1;
#pragma omp parallel for schedule(static) num_threads(n_threads)
#endif
    for (int64_t r = 0; r < n_rows; ++r)
        for (int64_t c = 0; c < n_cols; ++c)
            y[c * ldy + r] = orc_vec_dot_q6_K_q8_K((int) k, w + r * nb, xq + c * nb, order);
    (void) n_threads;
}

/* ======================================================================== */
/* Decode-stack helpers (RMSNorm is the reference's sme_ai_rmsnorm_f32,      */
/* sme_ai_ops.c:1060-1092: y = x / sqrt(mean(x^2) + eps)).  The sum of       */
/* squares is taken in the fixed order the GPU kernels use, so both sides    */
/* round identically:                                                        */
/*   1. per 32-value group g (values 32g .. 32g+31): the squares x*x, each   */
/*      rounded, folded pairwise at distances 16, 8, 4, 2, 1 -> s_g;         */
/*   2. 32 accumulators a_l = s_l + s_{l+32} + s_{l+64} + ... (ascending,    */
/*      starting from 0), folded pairwise at distances 16, 8, 4, 2, 1.       */
/* Step 1 is what one warp computes from one value per lane (the GEMV's row  */
/* group), step 2 what one warp computes from all the group sums.            */
/* ======================================================================== */
static float orc_fold32(float *a) {
    for (int width = 16; width >= 1; width /= 2)
        for (int l = 0; l < width; ++l) a[l] = a[l] + a[l + width];
    return a[0];
}

float orc_rms_group_sumsq(const float *x) {
    float a[32];
    for (int l = 0; l < 32; ++l) a[l] = x[l] * x[l];
    return orc_fold32(a);
}

float orc_rms_sumsq(const float *x, int64_t k) {
    int64_t groups = k / 32;
    float a[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int64_t g = l; g < groups; g += 32) acc = acc + orc_rms_group_sumsq(x + 32 * g);
        a[l] = acc;
    }
    return orc_fold32(a);
}

float orc_rms_inv(const float *x, int64_t k, float eps) {
    float mean = orc_rms_sumsq(x, k) / (float) k;
    return 1.0f / sqrtf(mean + eps);
}

/* With the reference's weight operand (sme_ai_ops.c:1084-1086): y = x * inv,
 * then y * weight[j] -- two multiplies, each rounded; weight NULL = none. */
void orc_rmsnorm_w_quantize_q8_K(const float *x, const float *weight, orc_block_q8_K *y, int64_t k, float eps,
                                 int rounding) {
    float inv = orc_rms_inv(x, k, eps);
    float *tmp = (float *) malloc((size_t) k * sizeof(float));
    for (int64_t i = 0; i < k; ++i) {
        tmp[i] = x[i] * inv;
        if (weight) tmp[i] = tmp[i] * weight[i];
    }
    orc_quantize_row_q8_K(tmp, y, k, rounding);
    free(tmp);
}

void orc_rmsnorm_quantize_q8_K(const float *x, orc_block_q8_K *y, int64_t k, float eps, int rounding) {
    orc_rmsnorm_w_quantize_q8_K(x, NULL, y, k, eps, rounding);
}

/* h = silu(g) * u with silu(g) = g / (1 + expf(-g)), sme_ai_ops.c:879-887
 * then :801-814. */
void orc_silu_mul(const float *g, const float *u, float *h, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        float s = g[i] / (1.0f + expf(-g[i]));
        h[i] = s * u[i];
    }
}
