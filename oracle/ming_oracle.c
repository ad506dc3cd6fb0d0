/*
 * ming_oracle.c — CPU restatement of ming-tts-serve's LM decode step and DiT
 * flow head. TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline); see
 * ming_oracle.h for what each function follows and for the parity status.
 *
 * Arithmetic: bf16 storage, f32 accumulation, bf16 rounding (round to nearest
 * even) at the points MLX rounds. OpenMP parallelises over output features.
 */
#include "ming_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* bf16                                                                 */
/* ------------------------------------------------------------------ */

float mo_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t mo_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float rb(float x) { return mo_bf16_to_f32(mo_f32_to_bf16(x)); }
/* Round per mode: identity in F32 mode. */
static inline float R(float x, int mode) { return mode == MO_MODE_F32 ? x : rb(x); }
static inline float bf(const uint16_t* p, int64_t i) { return mo_bf16_to_f32(p[i]); }

void mo_round_bf16(const float* x, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = mo_f32_to_bf16(x[i]);
}

static int g_threads = 0;
void mo_set_threads(int n) {
    g_threads = n;
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}
int mo_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------ */
/* MLX affine quantization layout                                       */
/* ------------------------------------------------------------------ */

/* Element j of a row sits in word j / (32/bits), at bit bits*(j % (32/bits)),
 * little end first (MLX QuantizedLinear packing). */
void mo_unpack(const uint32_t* q, int rows, int cols, int bits, uint8_t* codes) {
    const int per = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int words = cols / per;
    for (int r = 0; r < rows; r++)
        for (int c = 0; c < cols; c++)
            codes[(int64_t)r * cols + c] = (uint8_t)((q[(int64_t)r * words + c / per] >> (bits * (c % per))) & mask);
}

void mo_pack(const uint8_t* codes, int rows, int cols, int bits, uint32_t* q) {
    const int per = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int words = cols / per;
    for (int r = 0; r < rows; r++)
        for (int w = 0; w < words; w++) {
            uint32_t v = 0;
            for (int j = 0; j < per; j++) v |= ((uint32_t)codes[(int64_t)r * cols + w * per + j] & mask) << (bits * j);
            q[(int64_t)r * words + w] = v;
        }
}

/* w = scale * q + bias, evaluated in f32 as MLX's dequantize does. */
void mo_lin_row(const mo_lin* l, int row, float* out) {
    const int K = l->in;
    if (l->fmt == 16) {
        for (int k = 0; k < K; k++) out[k] = bf(l->w, (int64_t)row * K + k);
        return;
    }
    const int bits = l->fmt, per = 32 / bits, G = l->group;
    const uint32_t mask = (1u << bits) - 1u;
    const uint32_t* qr = l->q + (int64_t)row * (K / per);
    const int ng = K / G;
    for (int g = 0; g < ng; g++) {
        const float s = bf(l->scales, (int64_t)row * ng + g);
        const float b = bf(l->biases, (int64_t)row * ng + g);
        for (int j = 0; j < G; j++) {
            const int k = g * G + j;
            const uint32_t c = (qr[k / per] >> (bits * (k % per))) & mask;
            out[k] = s * (float)c + b;
        }
    }
}

void mo_lin_dequant(const mo_lin* l, float* out) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < l->out; r++) mo_lin_row(l, r, out + (int64_t)r * l->in);
}

/* acc[r][n] = post[r] * sum_k W[n][k] xf[r][k] + bias[n], all f32 (no rounding). */
static void lin_apply(const mo_lin* l, const float* xf, int rows, const float* post, float* acc) {
    const int N = l->out, K = l->in;
#pragma omp parallel
    {
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int n = 0; n < N; n++) {
            mo_lin_row(l, n, w);
            const float b = l->bias ? bf(l->bias, n) : 0.0f;
            for (int r = 0; r < rows; r++) {
                const float* x = xf + (int64_t)r * K;
                float s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0, s5 = 0, s6 = 0, s7 = 0;
                int k = 0;
                for (; k + 8 <= K; k += 8) {
                    s0 += w[k] * x[k];
                    s1 += w[k + 1] * x[k + 1];
                    s2 += w[k + 2] * x[k + 2];
                    s3 += w[k + 3] * x[k + 3];
                    s4 += w[k + 4] * x[k + 4];
                    s5 += w[k + 5] * x[k + 5];
                    s6 += w[k + 6] * x[k + 6];
                    s7 += w[k + 7] * x[k + 7];
                }
                float s = ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7));
                for (; k < K; k++) s += w[k] * x[k];
                acc[(int64_t)r * N + n] = (post ? s * post[r] : s) + b;
            }
        }
        free(w);
    }
}

void mo_linear(const mo_lin* l, const uint16_t* x, int rows, uint16_t* y, int mode) {
    const int N = l->out, K = l->in;
    float* xf = (float*)malloc(sizeof(float) * (size_t)rows * K);
    float* acc = (float*)malloc(sizeof(float) * (size_t)rows * N);
    for (int64_t i = 0; i < (int64_t)rows * K; i++) xf[i] = bf(x, i);
    lin_apply(l, xf, rows, NULL, acc);
    for (int64_t i = 0; i < (int64_t)rows * N; i++) y[i] = mo_f32_to_bf16(R(acc[i], mode));
    free(xf);
    free(acc);
}

/* ------------------------------------------------------------------ */
/* Norm-prologue linear: RMSNorm(x) then W.                              */
/* ------------------------------------------------------------------ */

/* Per-row 1/rms in f32: rsqrt(mean(x^2) + eps). */
static void row_inv_rms(const float* x, int rows, int K, float eps, float* inv) {
    for (int r = 0; r < rows; r++) {
        double ss = 0;
        for (int k = 0; k < K; k++) ss += (double)x[(int64_t)r * K + k] * x[(int64_t)r * K + k];
        inv[r] = 1.0f / sqrtf((float)(ss / K) + eps);
    }
}

/* acc = W rmsnorm(x) + bias (f32, not yet rounded) following `mode`:
 *   FUSED: x*nw in f32, 1/rms on the f32 sum (src/ming_fused.zig:100-142)
 *   GRAPH: normed row rounded: rb(rb(x*inv)*nw) (MLX fast_rms_norm)
 *   F32:   x*inv*nw unrounded. */
static void norm_linear(const mo_lin* l, const float* x, int rows, const uint16_t* nw, float eps, float* acc, int mode) {
    const int K = l->in;
    float* inv = (float*)malloc(sizeof(float) * (size_t)rows);
    float* xf = (float*)malloc(sizeof(float) * (size_t)rows * K);
    row_inv_rms(x, rows, K, eps, inv);
    for (int r = 0; r < rows; r++)
        for (int k = 0; k < K; k++) {
            const int64_t i = (int64_t)r * K + k;
            const float w = bf(nw, k);
            if (mode == MO_MODE_FUSED) xf[i] = x[i] * w;
            else if (mode == MO_MODE_GRAPH) xf[i] = rb(rb(x[i] * inv[r]) * w);
            else xf[i] = x[i] * inv[r] * w;
        }
    lin_apply(l, xf, rows, mode == MO_MODE_FUSED ? inv : NULL, acc);
    free(inv);
    free(xf);
}

/* MLX fast_rms_norm output: rb(w * rb(x * inv)). */
static void rms_norm_rows(const float* x, int rows, int K, const uint16_t* nw, float eps, float* out, int mode) {
    float* inv = (float*)malloc(sizeof(float) * (size_t)rows);
    row_inv_rms(x, rows, K, eps, inv);
    for (int r = 0; r < rows; r++)
        for (int k = 0; k < K; k++) {
            const int64_t i = (int64_t)r * K + k;
            out[i] = R(bf(nw, k) * R(x[i] * inv[r], mode), mode);
        }
    free(inv);
}

/* ------------------------------------------------------------------ */
/* Qwen2 LM (src/ming_model.zig:566-614; fused rounding src/ming_fused.zig:296-399) */
/* ------------------------------------------------------------------ */

static inline float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

static int lm_run(const mo_lm* m, mo_kv* kv, const uint16_t* x_in, int L, int layers_run, float* x /*[L][H] out*/, int mode) {
    const int H = m->hidden, NH = m->heads, NKV = m->kv_heads, D = m->head_dim, FF = m->ff;
    const int QD = NH * D, KD = NKV * D, grp = NH / NKV, half = D / 2;
    const int pos0 = kv->len;
    if (pos0 + L > kv->cap) return -1;
    for (int64_t i = 0; i < (int64_t)L * H; i++) x[i] = bf(x_in, i);
    float* q = (float*)malloc(sizeof(float) * (size_t)L * QD);
    float* k = (float*)malloc(sizeof(float) * (size_t)L * KD);
    float* v = (float*)malloc(sizeof(float) * (size_t)L * KD);
    float* att = (float*)malloc(sizeof(float) * (size_t)L * QD);
    float* tmp = (float*)malloc(sizeof(float) * (size_t)L * H);
    float* g = (float*)malloc(sizeof(float) * (size_t)L * FF);
    float* u = (float*)malloc(sizeof(float) * (size_t)L * FF);
    float* hh = (float*)malloc(sizeof(float) * (size_t)L * FF);
    const float log2th = log2f(m->theta);
    for (int li = 0; li < layers_run; li++) {
        const mo_lin* W = m->lin + (int64_t)li * 7;
        const uint16_t* ln1 = m->ln1 + (int64_t)li * H;
        const uint16_t* ln2 = m->ln2 + (int64_t)li * H;
        /* q/k/v: rms1 + linear + bias, rounded (LA; addmm) */
        norm_linear(&W[0], x, L, ln1, m->eps, q, mode);
        norm_linear(&W[1], x, L, ln1, m->eps, k, mode);
        norm_linear(&W[2], x, L, ln1, m->eps, v, mode);
        for (int64_t i = 0; i < (int64_t)L * QD; i++) q[i] = R(q[i], mode);
        for (int64_t i = 0; i < (int64_t)L * KD; i++) { k[i] = R(k[i], mode); v[i] = R(v[i], mode); }
        /* RoPE, non-traditional: pairs (d, d + D/2), inv_freq = exp2(-(d/half) * log2 theta),
         * angle = pos * inv_freq in f32, rotated in f32 and rounded once. */
        for (int r = 0; r < L; r++) {
            const float pos = (float)(pos0 + r);
            for (int d = 0; d < half; d++) {
                const float th = pos * exp2f(-((float)d / (float)half) * log2th);
                const float c = cosf(th), s = sinf(th);
                for (int h = 0; h < NH; h++) {
                    float* p = q + (int64_t)r * QD + h * D;
                    const float a = p[d], b = p[d + half];
                    p[d] = R(a * c - b * s, mode);
                    p[d + half] = R(a * s + b * c, mode);
                }
                for (int h = 0; h < NKV; h++) {
                    float* p = k + (int64_t)r * KD + h * D;
                    const float a = p[d], b = p[d + half];
                    p[d] = R(a * c - b * s, mode);
                    p[d + half] = R(a * s + b * c, mode);
                }
            }
        }
        /* KV append: cache layout [layer][kv head][pos][dim] */
        for (int r = 0; r < L; r++)
            for (int h = 0; h < NKV; h++)
                for (int d = 0; d < D; d++) {
                    const int64_t ci = (((int64_t)li * NKV + h) * kv->cap + pos0 + r) * D + d;
                    kv->k[ci] = k[(int64_t)r * KD + h * D + d];
                    kv->v[ci] = v[(int64_t)r * KD + h * D + d];
                }
        /* attention: row r at absolute position pos0+r attends to 0..pos0+r */
#pragma omp parallel for collapse(2) schedule(static)
        for (int r = 0; r < L; r++)
            for (int h = 0; h < NH; h++) {
                const int kh = h / grp, n = pos0 + r + 1;
                const float* qr = q + (int64_t)r * QD + h * D;
                float* sc = (float*)malloc(sizeof(float) * (size_t)n);
                float mx = -INFINITY;
                for (int j = 0; j < n; j++) {
                    const float* kr = kv->k + (((int64_t)li * NKV + kh) * kv->cap + j) * D;
                    float a = 0;
                    for (int d = 0; d < D; d++) a += (0.125f * qr[d]) * kr[d];
                    sc[j] = a;
                    if (a > mx) mx = a;
                }
                float sum = 0;
                for (int j = 0; j < n; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
                for (int d = 0; d < D; d++) {
                    float o = 0;
                    for (int j = 0; j < n; j++) o += sc[j] * kv->v[(((int64_t)li * NKV + kh) * kv->cap + j) * D + d];
                    att[(int64_t)r * QD + h * D + d] = R(o / sum, mode);
                }
                free(sc);
            }
        /* o_proj + residual: x1 = rb(x + rb(o W^T)) (LC) */
        lin_apply(&W[3], att, L, NULL, tmp);
        for (int64_t i = 0; i < (int64_t)L * H; i++) x[i] = R(x[i] + R(tmp[i], mode), mode);
        /* rms2 + gate/up + swiglu: h = rb(rb(g * rb(sigmoid g)) * u) (LD) */
        norm_linear(&W[4], x, L, ln2, m->eps, g, mode);
        norm_linear(&W[5], x, L, ln2, m->eps, u, mode);
        for (int64_t i = 0; i < (int64_t)L * FF; i++) {
            const float gg = R(g[i], mode), uu = R(u[i], mode);
            hh[i] = R(R(gg * R(sigmoidf_(gg), mode), mode) * uu, mode);
        }
        /* down + residual (LE) */
        lin_apply(&W[6], hh, L, NULL, tmp);
        for (int64_t i = 0; i < (int64_t)L * H; i++) x[i] = R(x[i] + R(tmp[i], mode), mode);
    }
    kv->len = pos0 + L;
    free(q); free(k); free(v); free(att); free(tmp); free(g); free(u); free(hh);
    return 0;
}

void mo_stop_prob(const mo_lm* m, const uint16_t* z, int rows, float* p, int mode) {
    /* softmax(stop_head(z).astype(f32))[1]: the logits are rounded to bf16 first. */
    float* xf = (float*)malloc(sizeof(float) * (size_t)rows * m->hidden);
    float logits[2 * 64];
    for (int64_t i = 0; i < (int64_t)rows * m->hidden; i++) xf[i] = bf(z, i);
    for (int r0 = 0; r0 < rows; r0 += 64) {
        const int n = rows - r0 < 64 ? rows - r0 : 64;
        lin_apply(&m->stop, xf + (int64_t)r0 * m->hidden, n, NULL, logits);
        for (int r = 0; r < n; r++) {
            const float l0 = R(logits[r * 2], mode), l1 = R(logits[r * 2 + 1], mode);
            const float mx = l0 > l1 ? l0 : l1;
            const float e0 = expf(l0 - mx), e1 = expf(l1 - mx);
            p[r0 + r] = e1 / (e0 + e1);
        }
    }
    free(xf);
}

int mo_lm_forward(const mo_lm* m, mo_kv* kv, const uint16_t* x, int L, uint16_t* out, float* stop, int mode) {
    const int H = m->hidden;
    float* xs = (float*)malloc(sizeof(float) * (size_t)L * H);
    float* zn = (float*)malloc(sizeof(float) * (size_t)L * H);
    if (lm_run(m, kv, x, L, m->layers, xs, mode) != 0) { free(xs); free(zn); return -1; }
    rms_norm_rows(xs, L, H, m->norm, m->eps, zn, mode);
    for (int64_t i = 0; i < (int64_t)L * H; i++) out[i] = mo_f32_to_bf16(zn[i]);
    if (stop) mo_stop_prob(m, out, L, stop, mode);
    free(xs);
    free(zn);
    return 0;
}

int mo_lm_forward_f32(const mo_lm* m, mo_kv* kv, const uint16_t* x, int L, float* out, int mode) {
    const int H = m->hidden;
    float* xs = (float*)malloc(sizeof(float) * (size_t)L * H);
    if (lm_run(m, kv, x, L, m->layers, xs, mode) != 0) { free(xs); return -1; }
    rms_norm_rows(xs, L, H, m->norm, m->eps, out, mode);
    free(xs);
    return 0;
}

int mo_lm_forward_partial(const mo_lm* m, mo_kv* kv, const uint16_t* x, int L, int layers_run, uint16_t* out, int mode) {
    const int H = m->hidden;
    float* xs = (float*)malloc(sizeof(float) * (size_t)L * H);
    if (lm_run(m, kv, x, L, layers_run, xs, mode) != 0) { free(xs); return -1; }
    for (int64_t i = 0; i < (int64_t)L * H; i++) out[i] = mo_f32_to_bf16(xs[i]);
    free(xs);
    return 0;
}

/* ------------------------------------------------------------------ */
/* DiT blocks, token conditioning (src/ming_model.zig:770-797;           */
/* fused kernels A-D, src/ming_fused.zig:144-245)                        */
/* ------------------------------------------------------------------ */

/* mlx.nn.gelu_approx with every bf16 op rounded, constants as bf16 weak scalars
 * (src/ming_model.zig:855-862; src/ming_fused.zig:229-236). */
static inline float gelu_chain(float x, int mode) {
    const float c1 = R(0.044715f, mode), c2 = R(0.7978845608f, mode);
    const float x3 = R(x * x * x, mode);
    const float inner = R(x + R(c1 * x3, mode), mode);
    const float th = R(tanhf(R(c2 * inner, mode)), mode);
    return R(R(0.5f * x, mode) * R(1.0f + th, mode), mode);
}

/* Interleaved-pair rotary (x_transformers style): pairs (2i, 2i+1), angle =
 * pos * inv_freq[i] in f32, rotated in f32 from the rounded q/k, rounded once. */
static void rotary_interleaved(float* p, int heads, int D, int pos, const float* inv_freq, int mode) {
    for (int h = 0; h < heads; h++)
        for (int i = 0; i < D / 2; i++) {
            const float f = (float)pos * inv_freq[i];
            const float c = cosf(f), s = sinf(f);
            float* e = p + h * D + 2 * i;
            const float a = e[0], b = e[1];
            e[0] = R(a * c - b * s, mode);
            e[1] = R(a * s + b * c, mode);
        }
}

/* Attention of R = B*L rows over their own L positions (no mask), scale 1/8. */
static void seq_attention(const float* q, const float* k, const float* v, int B, int L, int heads, int D, float* out, int mode) {
    const int W = heads * D;
    for (int b = 0; b < B; b++)
        for (int i = 0; i < L; i++)
            for (int h = 0; h < heads; h++) {
                float sc[64];
                float mx = -INFINITY;
                const float* qr = q + ((int64_t)b * L + i) * W + h * D;
                for (int j = 0; j < L; j++) {
                    const float* kr = k + ((int64_t)b * L + j) * W + h * D;
                    float a = 0;
                    for (int d = 0; d < D; d++) a += (0.125f * qr[d]) * kr[d];
                    sc[j] = a;
                    if (a > mx) mx = a;
                }
                float sum = 0;
                for (int j = 0; j < L; j++) { sc[j] = expf(sc[j] - mx); sum += sc[j]; }
                for (int d = 0; d < D; d++) {
                    float o = 0;
                    for (int j = 0; j < L; j++) o += sc[j] * v[((int64_t)b * L + j) * W + h * D + d];
                    out[((int64_t)b * L + i) * W + h * D + d] = R(o / sum, mode);
                }
            }
}

static void dit_block_tok(const mo_dit* d, int blk, float* x, int B, int L, int mode) {
    const int H = d->hidden, NR = B * L, FF = d->ff;
    const mo_lin* W = d->lin + (int64_t)blk * 6;
    const uint16_t* n1 = d->norm1 + (int64_t)blk * H;
    const uint16_t* n2 = d->norm2 + (int64_t)blk * H;
    float* q = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* k = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* v = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* att = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* tmp = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* f1 = (float*)malloc(sizeof(float) * (size_t)NR * FF);
    norm_linear(&W[0], x, NR, n1, 1e-6f, q, mode);
    norm_linear(&W[1], x, NR, n1, 1e-6f, k, mode);
    norm_linear(&W[2], x, NR, n1, 1e-6f, v, mode);
    for (int64_t i = 0; i < (int64_t)NR * H; i++) { q[i] = R(q[i], mode); k[i] = R(k[i], mode); v[i] = R(v[i], mode); }
    for (int r = 0; r < NR; r++) {
        rotary_interleaved(q + (int64_t)r * H, d->heads, d->head_dim, r % L, d->inv_freq, mode);
        rotary_interleaved(k + (int64_t)r * H, d->heads, d->head_dim, r % L, d->inv_freq, mode);
    }
    seq_attention(q, k, v, B, L, d->heads, d->head_dim, att, mode);
    lin_apply(&W[3], att, NR, NULL, tmp);
    for (int64_t i = 0; i < (int64_t)NR * H; i++) x[i] = R(x[i] + R(tmp[i], mode), mode);
    norm_linear(&W[4], x, NR, n2, 1e-6f, f1, mode);
    for (int64_t i = 0; i < (int64_t)NR * FF; i++) f1[i] = gelu_chain(R(f1[i], mode), mode);
    lin_apply(&W[5], f1, NR, NULL, tmp);
    for (int64_t i = 0; i < (int64_t)NR * H; i++) x[i] = R(x[i] + R(tmp[i], mode), mode);
    free(q); free(k); free(v); free(att); free(tmp); free(f1);
}

void mo_dit_forward(const mo_dit* d, const uint16_t* x_in, int B, int L, uint16_t* out, int mode) {
    const int64_t n = (int64_t)B * L * d->hidden;
    float* x = (float*)malloc(sizeof(float) * (size_t)n);
    for (int64_t i = 0; i < n; i++) x[i] = bf(x_in, i);
    for (int b = 0; b < d->blocks; b++) dit_block_tok(d, b, x, B, L, mode);
    for (int64_t i = 0; i < n; i++) out[i] = mo_f32_to_bf16(x[i]);
    free(x);
}

/* ------------------------------------------------------------------ */
/* Flow head (src/ming_model.zig:966-992,1064-1091,1159-1215)            */
/* ------------------------------------------------------------------ */

#define FLOW_STEPS 10

/* EPSS + sway schedule in bf16 (flowSchedule, src/ming_model.zig:1205-1215):
 * t = (1/32) * sched; t = t + (-1) * (cos(pi/2 * t) - 1 + t); then per step
 * dt = t[i+1] - t[i] and sq = |dt| ** 0.5, each op rounded to bf16. */
/* The schedule is computed in the noise dtype: bf16 (every op rounded), or
 * f32 in F32 mode. */
static void flow_schedule_mode(float* t, float* dt, float* sq, int mode) {
    static const float sched[FLOW_STEPS + 1] = {0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32};
    const float h = R(1.0f / 32.0f, mode), hp = R(3.14159265358979f / 2.0f, mode), one = 1.0f;
    for (int i = 0; i <= FLOW_STEPS; i++) {
        float tt = R(h * R(sched[i], mode), mode);
        const float ct = R(cosf(R(hp * tt, mode)), mode);
        const float sw = R(R(ct - one, mode) + tt, mode);
        t[i] = R(tt + R(-1.0f * sw, mode), mode);
    }
    for (int i = 0; i < FLOW_STEPS; i++) {
        dt[i] = R(t[i + 1] - t[i], mode);
        sq[i] = R(powf(fabsf(dt[i]), 0.5f), mode);
    }
}

void mo_flow_schedule(float* t, float* dt, float* sq) { flow_schedule_mode(t, dt, sq, MO_MODE_FUSED); }

/* TimestepEmbedder (src/ming_model.zig:1064-1076): sinusoid of rb(1000*t)
 * with freq exp(-ln(1e4) k / 127), [sin, cos] rounded, Linear, SiLU (rounded
 * per op), Linear. t_freq is built as in Model.load (:966-975). */
static void timestep_embed(const mo_lin* mlp0, const mo_lin* mlp2, int freq_dim, const float* t, int n, float* out, int mode) {
    const int half = freq_dim / 2, H = mlp0->out;
    const float e = (float)(log(10000.0) / (double)(half - 1));
    float* sincos = (float*)malloc(sizeof(float) * (size_t)n * freq_dim);
    float* h0 = (float*)malloc(sizeof(float) * (size_t)n * H);
    for (int r = 0; r < n; r++) {
        const float ts = R(R(1000.0f, mode) * t[r], mode);
        for (int j = 0; j < half; j++) {
            const float f = expf((float)j * -e);
            const float a = ts * f;
            sincos[(int64_t)r * freq_dim + j] = R(sinf(a), mode);
            sincos[(int64_t)r * freq_dim + half + j] = R(cosf(a), mode);
        }
    }
    lin_apply(mlp0, sincos, n, NULL, h0);
    for (int64_t i = 0; i < (int64_t)n * H; i++) {
        const float a = R(h0[i], mode);
        h0[i] = R(a * R(sigmoidf_(a), mode), mode);
    }
    lin_apply(mlp2, h0, n, NULL, out);
    for (int64_t i = 0; i < (int64_t)n * H; i++) out[i] = R(out[i], mode);
    free(sincos);
    free(h0);
}

void mo_flow_temb(const mo_flow* f, uint16_t* te, int mode) {
    float t[FLOW_STEPS + 1], dt[FLOW_STEPS], sq[FLOW_STEPS];
    flow_schedule_mode(t, dt, sq, mode);
    float* o = (float*)malloc(sizeof(float) * (size_t)FLOW_STEPS * f->dit.hidden);
    timestep_embed(&f->t_mlp0, &f->t_mlp2, f->t_mlp0.in, t, FLOW_STEPS, o, mode);
    for (int64_t i = 0; i < (int64_t)FLOW_STEPS * f->dit.hidden; i++) te[i] = mo_f32_to_bf16(o[i]);
    free(o);
}

/* Final RMSNorm + linear on one row, as the fused kernel F folds it
 * (src/ming_fused.zig:263-289) or as MLX's rms + addmm (GRAPH/F32). */
static void final_row(const mo_lin* fl, const uint16_t* nw, const float* x, int K, float* out, int mode) {
    float acc[256];
    if (mode == MO_MODE_FUSED) {
        double ss = 0;
        for (int k = 0; k < K; k++) ss += (double)x[k] * x[k];
        const float inv = 1.0f / sqrtf((float)(ss / K) + 1e-6f);
        float* w = (float*)malloc(sizeof(float) * (size_t)K);
        for (int o = 0; o < fl->out; o++) {
            mo_lin_row(fl, o, w);
            float a = 0;
            for (int k = 0; k < K; k++) a += (w[k] * bf(nw, k)) * x[k];
            out[o] = a * inv + (fl->bias ? bf(fl->bias, o) : 0.0f);
        }
        free(w);
    } else {
        float* hn = (float*)malloc(sizeof(float) * (size_t)K);
        rms_norm_rows(x, 1, K, nw, 1e-6f, hn, mode);
        lin_apply(fl, hn, 1, NULL, acc);
        for (int o = 0; o < fl->out; o++) out[o] = acc[o];
        free(hn);
    }
}

/* CFG combine + Euler update for one latent channel (kernel F epilogue). */
static inline float cfg_euler(float y, float pc, float pu, float cfg, float dtv, float shift, float sqv, float sde, int mode) {
    const float f0 = R(pc + R(R(pc - pu, mode) * R(cfg, mode), mode), mode);
    float yn = R(y + R(dtv * f0, mode), mode);
    if (shift != 0.0f) yn = R(yn + R(R(R(shift, mode) * sqv, mode) * sde, mode), mode);
    return yn;
}

void mo_cfm_steps(const mo_flow* f, const uint16_t* z, const uint16_t* hist, const uint16_t* y_in,
                  const uint16_t* sde, float cfg, float shift, int step0, int nsteps, uint16_t* y_out, int mode) {
    const int H = f->dit.hidden, LAT = f->latent, CD = f->cond_dim, L = 3;
    float t[FLOW_STEPS + 1], dt[FLOW_STEPS], sq[FLOW_STEPS];
    flow_schedule_mode(t, dt, sq, mode);
    float* te = (float*)malloc(sizeof(float) * (size_t)FLOW_STEPS * H);
    timestep_embed(&f->t_mlp0, &f->t_mlp2, f->t_mlp0.in, t, FLOW_STEPS, te, mode);
    /* fixed across the Euler steps: c_emb of [z, 0] and x_emb(hist) */
    float* zc = (float*)calloc((size_t)2 * CD, sizeof(float));
    for (int i = 0; i < CD; i++) zc[i] = bf(z, i);
    float* ce = (float*)malloc(sizeof(float) * (size_t)2 * H);
    lin_apply(&f->c_emb, zc, 2, NULL, ce);
    float hf[256], yv[256], xe[1 << 12];
    for (int i = 0; i < LAT; i++) { hf[i] = bf(hist, i); yv[i] = bf(y_in, i); }
    float* xh = (float*)malloc(sizeof(float) * (size_t)H);
    lin_apply(&f->x_emb, hf, 1, NULL, xh);
    for (int i = 0; i < H; i++) { xh[i] = R(xh[i], mode); ce[i] = R(ce[i], mode); ce[H + i] = R(ce[H + i], mode); }
    float* rows = (float*)malloc(sizeof(float) * (size_t)2 * L * H);
    for (int s = step0; s < step0 + nsteps && s < FLOW_STEPS; s++) {
        lin_apply(&f->x_emb, yv, 1, NULL, xe);
        for (int b = 0; b < 2; b++)
            for (int i = 0; i < H; i++) {
                rows[((int64_t)b * L + 0) * H + i] = R(te[(int64_t)s * H + i] + ce[(int64_t)b * H + i], mode);
                rows[((int64_t)b * L + 1) * H + i] = xh[i];
                rows[((int64_t)b * L + 2) * H + i] = R(xe[i], mode);
            }
        for (int blk = 0; blk < f->dit.blocks; blk++) dit_block_tok(&f->dit, blk, rows, 2, L, mode);
        float pc[256], pu[256];
        final_row(&f->final_lin, f->final_norm, rows + (int64_t)(L - 1) * H, H, pc, mode);
        final_row(&f->final_lin, f->final_norm, rows + (int64_t)(2 * L - 1) * H, H, pu, mode);
        for (int o = 0; o < LAT; o++) {
            const float sv = sde ? bf(sde, (int64_t)s * LAT + o) : 0.0f;
            yv[o] = cfg_euler(yv[o], R(pc[o], mode), R(pu[o], mode), cfg, dt[s], shift, sq[s], sv, mode);
        }
    }
    for (int o = 0; o < LAT; o++) y_out[o] = mo_f32_to_bf16(yv[o]);
    free(te); free(zc); free(ce); free(xh); free(rows);
}

void mo_cfm_sample(const mo_flow* f, const uint16_t* z, const uint16_t* hist, const uint16_t* noise,
                   const uint16_t* sde, float cfg, float shift, uint16_t* y_out, int mode) {
    mo_cfm_steps(f, z, hist, noise, sde, cfg, shift, 0, FLOW_STEPS, y_out, mode);
}

/* Aggregator (src/ming_model.zig:1040-1053): x_embedder, CLS row prepended,
 * DiT stack at L = 2, final RMSNorm + linear on the CLS row. */
void mo_aggregate(const mo_agg* a, const uint16_t* latent, int B, uint16_t* out, int mode) {
    const int H = a->dit.hidden, LAT = a->x_emb.in, NO = a->final_lin.out;
    float* lf = (float*)malloc(sizeof(float) * (size_t)B * LAT);
    float* xe = (float*)malloc(sizeof(float) * (size_t)B * H);
    float* rows = (float*)malloc(sizeof(float) * (size_t)B * 2 * H);
    float* o = (float*)malloc(sizeof(float) * (size_t)NO);
    float* hn = (float*)malloc(sizeof(float) * (size_t)H);
    for (int64_t i = 0; i < (int64_t)B * LAT; i++) lf[i] = bf(latent, i);
    lin_apply(&a->x_emb, lf, B, NULL, xe);
    for (int b = 0; b < B; b++)
        for (int i = 0; i < H; i++) {
            rows[((int64_t)b * 2 + 0) * H + i] = bf(a->cls, i);
            rows[((int64_t)b * 2 + 1) * H + i] = R(xe[(int64_t)b * H + i], mode);
        }
    for (int blk = 0; blk < a->dit.blocks; blk++) dit_block_tok(&a->dit, blk, rows, B, 2, mode);
    /* the final layer is MLX rms + addmm in every mode */
    const int fm = mode == MO_MODE_F32 ? MO_MODE_F32 : MO_MODE_GRAPH;
    for (int b = 0; b < B; b++) {
        rms_norm_rows(rows + (int64_t)b * 2 * H, 1, H, a->final_norm, 1e-6f, hn, fm);
        lin_apply(&a->final_lin, hn, 1, NULL, o);
        for (int i = 0; i < NO; i++) out[(int64_t)b * NO + i] = mo_f32_to_bf16(R(o[i], fm));
    }
    free(lf); free(xe); free(rows); free(o); free(hn);
}

/* ------------------------------------------------------------------ */
/* adaLN-Zero DiT head (the benchmark's flow head; no reference code). */
/* Pinned choices: LayerNorm without affine (eps 1e-6); modulation        */
/* h = LN(x) * (1 + scale) + shift; gated residuals; SiLU(c) feeds every */
/* modulation linear; interleaved rotary over the frame positions; CFG   */
/* with the condition zeroed; the reference's schedule and Euler update. */
/* FUSED mode evaluates the modulation in f32 and rounds once (the GPU   */
/* prologue); GRAPH mode rounds every op.                                */
/* ------------------------------------------------------------------ */

static void ln_modulate(const float* x, int rows, int H, const float* shift, const float* scale, int mod_stride, int rows_per_mod,
                        float* out, int mode) {
    for (int r = 0; r < rows; r++) {
        const float* xr = x + (int64_t)r * H;
        double mu = 0, var = 0;
        for (int i = 0; i < H; i++) mu += xr[i];
        mu /= H;
        for (int i = 0; i < H; i++) var += (xr[i] - mu) * (xr[i] - mu);
        var /= H;
        const float inv = 1.0f / sqrtf((float)var + 1e-6f);
        const float* sh = shift + (int64_t)(r / rows_per_mod) * mod_stride;
        const float* sc = scale + (int64_t)(r / rows_per_mod) * mod_stride;
        for (int i = 0; i < H; i++) {
            const float n = (xr[i] - (float)mu) * inv;
            if (mode == MO_MODE_FUSED) out[(int64_t)r * H + i] = rb(n * (1.0f + sc[i]) + sh[i]);
            else out[(int64_t)r * H + i] = R(R(R(n, mode) * R(1.0f + sc[i], mode), mode) + sh[i], mode);
        }
    }
}

void mo_ada_temb(const mo_ada* a, uint16_t* te, int mode) {
    float t[FLOW_STEPS + 1], dt[FLOW_STEPS], sq[FLOW_STEPS];
    flow_schedule_mode(t, dt, sq, mode);
    float* o = (float*)malloc(sizeof(float) * (size_t)FLOW_STEPS * a->hidden);
    timestep_embed(&a->t_mlp0, &a->t_mlp2, a->freq_dim, t, FLOW_STEPS, o, mode);
    for (int64_t i = 0; i < (int64_t)FLOW_STEPS * a->hidden; i++) te[i] = mo_f32_to_bf16(o[i]);
    free(o);
}

void mo_ada_steps(const mo_ada* a, int B, const uint16_t* z, const uint16_t* y_in, const uint16_t* sde,
                  float cfg, float shift, int step0, int nsteps, uint16_t* y_out, int mode) {
    const int H = a->hidden, F = a->frames, LAT = a->latent, CD = a->cond_dim, FF = a->ff;
    const int NC = 2 * B;        /* condition rows: cond halves then uncond halves */
    const int NR = NC * F;       /* token rows */
    float t[FLOW_STEPS + 1], dt[FLOW_STEPS], sq[FLOW_STEPS];
    flow_schedule_mode(t, dt, sq, mode);
    float* te = (float*)malloc(sizeof(float) * (size_t)FLOW_STEPS * H);
    timestep_embed(&a->t_mlp0, &a->t_mlp2, a->freq_dim, t, FLOW_STEPS, te, mode);
    /* c_emb of [z_b ..., 0 ...] */
    float* zc = (float*)calloc((size_t)NC * CD, sizeof(float));
    for (int64_t i = 0; i < (int64_t)B * CD; i++) zc[i] = bf(z, i);
    float* ce = (float*)malloc(sizeof(float) * (size_t)NC * H);
    lin_apply(&a->c_emb, zc, NC, NULL, ce);
    for (int64_t i = 0; i < (int64_t)NC * H; i++) ce[i] = R(ce[i], mode);
    float* y = (float*)malloc(sizeof(float) * (size_t)B * F * LAT);
    for (int64_t i = 0; i < (int64_t)B * F * LAT; i++) y[i] = bf(y_in, i);
    float* sc = (float*)malloc(sizeof(float) * (size_t)NC * H);
    float* mod = (float*)malloc(sizeof(float) * (size_t)NC * 6 * H);
    float* x = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* hm = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* q = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* k = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* v = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* att = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* tmp = (float*)malloc(sizeof(float) * (size_t)NR * H);
    float* f1 = (float*)malloc(sizeof(float) * (size_t)NR * FF);
    float* yin = (float*)malloc(sizeof(float) * (size_t)NR * LAT);
    float* vel = (float*)malloc(sizeof(float) * (size_t)NR * LAT);
    for (int s = step0; s < step0 + nsteps && s < FLOW_STEPS; s++) {
        /* c = rb(t_emb + c_emb); SiLU per op */
        for (int r = 0; r < NC; r++)
            for (int i = 0; i < H; i++) {
                const float c = R(te[(int64_t)s * H + i] + ce[(int64_t)r * H + i], mode);
                sc[(int64_t)r * H + i] = R(c * R(sigmoidf_(c), mode), mode);
            }
        /* token rows: both halves see the same latent y_b */
        for (int r = 0; r < NC; r++)
            for (int f = 0; f < F; f++)
                for (int j = 0; j < LAT; j++) yin[((int64_t)r * F + f) * LAT + j] = y[((int64_t)(r % B) * F + f) * LAT + j];
        lin_apply(&a->x_emb, yin, NR, NULL, x);
        for (int64_t i = 0; i < (int64_t)NR * H; i++) x[i] = R(x[i], mode);
        for (int blk = 0; blk < a->blocks; blk++) {
            const mo_lin* W = a->lin + (int64_t)blk * 7;
            lin_apply(&W[0], sc, NC, NULL, mod);
            for (int64_t i = 0; i < (int64_t)NC * 6 * H; i++) mod[i] = R(mod[i], mode);
            const int MS = 6 * H;
            /* attention branch: shift1 = mod[0:H], scale1 = mod[H:2H], gate1 = mod[2H:3H] */
            ln_modulate(x, NR, H, mod + 0, mod + H, MS, F, hm, mode);
            lin_apply(&W[1], hm, NR, NULL, q);
            lin_apply(&W[2], hm, NR, NULL, k);
            lin_apply(&W[3], hm, NR, NULL, v);
            for (int64_t i = 0; i < (int64_t)NR * H; i++) { q[i] = R(q[i], mode); k[i] = R(k[i], mode); v[i] = R(v[i], mode); }
            for (int r = 0; r < NR; r++) {
                rotary_interleaved(q + (int64_t)r * H, a->heads, a->head_dim, r % F, a->inv_freq, mode);
                rotary_interleaved(k + (int64_t)r * H, a->heads, a->head_dim, r % F, a->inv_freq, mode);
            }
            seq_attention(q, k, v, NC, F, a->heads, a->head_dim, att, mode);
            lin_apply(&W[4], att, NR, NULL, tmp);
            for (int r = 0; r < NR; r++)
                for (int i = 0; i < H; i++) {
                    const float g1 = mod[(int64_t)(r / F) * MS + 2 * H + i];
                    const int64_t xi = (int64_t)r * H + i;
                    x[xi] = R(x[xi] + R(g1 * R(tmp[xi], mode), mode), mode);
                }
            /* MLP branch: shift2 = mod[3H:4H], scale2 = mod[4H:5H], gate2 = mod[5H:6H] */
            ln_modulate(x, NR, H, mod + 3 * H, mod + 4 * H, MS, F, hm, mode);
            lin_apply(&W[5], hm, NR, NULL, f1);
            for (int64_t i = 0; i < (int64_t)NR * FF; i++) f1[i] = gelu_chain(R(f1[i], mode), mode);
            lin_apply(&W[6], f1, NR, NULL, tmp);
            for (int r = 0; r < NR; r++)
                for (int i = 0; i < H; i++) {
                    const float g2 = mod[(int64_t)(r / F) * MS + 5 * H + i];
                    const int64_t xi = (int64_t)r * H + i;
                    x[xi] = R(x[xi] + R(g2 * R(tmp[xi], mode), mode), mode);
                }
        }
        /* final: (shift, scale) = final_ada(SiLU c); LN-modulate; linear -> latent */
        lin_apply(&a->final_ada, sc, NC, NULL, mod);
        for (int64_t i = 0; i < (int64_t)NC * 2 * H; i++) mod[i] = R(mod[i], mode);
        ln_modulate(x, NR, H, mod + 0, mod + H, 2 * H, F, hm, mode);
        lin_apply(&a->final_lin, hm, NR, NULL, vel);
        /* CFG + Euler per (b, frame, channel) */
        for (int b = 0; b < B; b++)
            for (int f = 0; f < F; f++)
                for (int o = 0; o < LAT; o++) {
                    const float pc = R(vel[((int64_t)b * F + f) * LAT + o], mode);
                    const float pu = R(vel[((int64_t)(B + b) * F + f) * LAT + o], mode);
                    const int64_t yi = ((int64_t)b * F + f) * LAT + o;
                    const float sv = sde ? bf(sde, (int64_t)s * B * F * LAT + yi) : 0.0f;
                    y[yi] = cfg_euler(y[yi], pc, pu, cfg, dt[s], shift, sq[s], sv, mode);
                }
    }
    for (int64_t i = 0; i < (int64_t)B * F * LAT; i++) y_out[i] = mo_f32_to_bf16(y[i]);
    free(te); free(zc); free(ce); free(y); free(sc); free(mod); free(x); free(hm);
    free(q); free(k); free(v); free(att); free(tmp); free(f1); free(yin); free(vel);
}

void mo_ada_sample(const mo_ada* a, int B, const uint16_t* z, const uint16_t* noise, const uint16_t* sde,
                   float cfg, float shift, uint16_t* y_out, int mode) {
    mo_ada_steps(a, B, z, noise, sde, cfg, shift, 0, FLOW_STEPS, y_out, mode);
}
