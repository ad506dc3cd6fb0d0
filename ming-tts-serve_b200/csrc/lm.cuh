// lm.cuh — the Qwen2 LM step (decode of B rows, or a prefill of L rows of one
// sequence) on the tiled linear kernel plus split-K paged attention.
//
// Per layer (the reference's five fused dispatches LA..LE,
// src/ming_fused.zig:296-399, re-cut for B200):
//   1. QKV      linear, RMSNorm prologue, epilogue: bias, bf16, RoPE (pairs
//               d, d+32), q to a row buffer, k/v appended to the paged cache.
//   2. attention split-K over 256-position splits of the paged cache
//               (GQA: one CTA serves the 7 query heads of one kv head).
//   3. O        linear, prologue combines the splits, epilogue residual.
//   4. gate/up  linear, RMSNorm prologue, epilogue SwiGLU (tile rows r/r+8 =
//               gate/up of one feature).
//   5. down     linear, epilogue residual.
// then the final RMSNorm + stop head.
#pragma once

#include <cuda.h>

#include "linear.cuh"

namespace ming {

constexpr int PAGE = 16;        // positions per KV page
constexpr int HD = 64;          // head dim (the kernels are written for 64)
constexpr int ATT_SPLIT = 256;  // positions per attention split
constexpr int PART_STRIDE = 2 + HD;  // m, l, acc[64] per (row, split, head)

// The paged KV pool: page-major, one page holds PAGE positions of every layer:
// [page][layer][K|V][kv_head][slot 0..15][dim 0..63] bf16.
struct KvDev {
    uint16_t* pool;
    const int* bt;  // block table [max_seqs][bt_ld] -> physical page
    int bt_ld, layers, kv_heads;
};
MING_DEV size_t kv_index(const KvDev& kv, int page, int layer, int which, int h, int slot) {
    return ((((size_t)page * kv.layers + layer) * 2 + which) * kv.kv_heads + h) * (PAGE * HD) + (size_t)slot * HD;
}

// Rows of the current batch: row r is sequence row_seq[r] at position row_pos[r].
struct RowsDev {
    const int* seq;
    const int* pos;
};

// Tile layout of the fused q|k|v linear: tile t covers head t/4 of its block,
// dims d0 = 8*(t%4) .. +7 (rows 0..7) and the RoPE partners d0+32.. (rows 8..15).
struct EpiQKV {
    const float* bias;
    uint16_t* q;  // [rows][heads*64]
    KvDev kv;
    RowsDev rows;
    int layer, heads, kv_heads;
    float log2_theta;
    MING_DEV void operator()(int tile, int r8, int row, float lo, float hi) const {
        const int qt = heads * 4, kt = kv_heads * 4;
        const int which = tile < qt ? 0 : (tile < qt + kt ? 1 : 2);
        const int lt = which == 0 ? tile : (which == 1 ? tile - qt : tile - qt - kt);
        const int h = lt >> 2, d = (lt & 3) * 8 + r8;
        float x1 = rb(lo + bias[tile * 16 + r8]);
        float x2 = rb(hi + bias[tile * 16 + r8 + 8]);
        const int pos = rows.pos[row], seq = which ? rows.seq[row] : 0;
        if (which < 2) {
            // MLX fast_rope (non-traditional): angle = pos * 2^(-(d/32) log2 theta), f32
            const float th = (float)pos * exp2f(-((float)d / 32.0f) * log2_theta);
            float s, c;
            sincosf(th, &s, &c);
            const float a = x1 * c - x2 * s, b = x1 * s + x2 * c;
            x1 = a;
            x2 = b;
        }
        if (which == 0) {
            uint16_t* qr = q + (size_t)row * heads * HD + h * HD;
            qr[d] = f2bf(x1);
            qr[d + 32] = f2bf(x2);
        } else {
            const int page = kv.bt[(size_t)seq * kv.bt_ld + pos / PAGE];
            uint16_t* dst = kv.pool + kv_index(kv, page, layer, which - 1, h, pos % PAGE);
            dst[d] = f2bf(x1);
            dst[d + 32] = f2bf(x2);
        }
    }
};

// Combines the attention splits of each row into the o_proj input:
// o = sum_s acc_s e^(m_s - M) / sum_s l_s e^(m_s - M), rounded to bf16 (the
// reference rounds the attention output, src/ming_fused.zig:373).
struct ProAttn {
    const float* part;  // [rows][nsplit_max][heads][PART_STRIDE]
    RowsDev rows;
    int nsplit_max, heads;
    int r0;
    float* st;  // [row][heads][2]: M, 1/L
    MING_DEV void init(int r0_, int nrows, float* aux) {
        r0 = r0_;
        st = aux;
        for (int e = threadIdx.x; e < nrows * heads; e += LIN_THREADS) {
            const int r = e / heads, h = e % heads, ar = r0 + r;
            const int ns = (rows.pos[ar] + 1 + ATT_SPLIT - 1) / ATT_SPLIT;
            float M = -INFINITY;
            for (int s = 0; s < ns; s++) M = fmaxf(M, part[(((size_t)ar * nsplit_max + s) * heads + h) * PART_STRIDE]);
            float L = 0.f;
            for (int s = 0; s < ns; s++) {
                const float* p = part + (((size_t)ar * nsplit_max + s) * heads + h) * PART_STRIDE;
                L += p[1] * expf(p[0] - M);
            }
            aux[(r * heads + h) * 2] = M;
            aux[(r * heads + h) * 2 + 1] = 1.0f / L;
        }
    }
    MING_DEV float y(int row, int k) const {
        const int ar = r0 + row, h = k / HD, d = k % HD;
        const int ns = (rows.pos[ar] + 1 + ATT_SPLIT - 1) / ATT_SPLIT;
        const float M = st[(row * heads + h) * 2], il = st[(row * heads + h) * 2 + 1];
        float o = 0.f;
        for (int s = 0; s < ns; s++) {
            const float* p = part + (((size_t)ar * nsplit_max + s) * heads + h) * PART_STRIDE;
            o += p[2 + d] * expf(p[0] - M);
        }
        return rb(o * il);
    }
    MING_DEV float post(int) const { return 1.f; }
};

// gate/up tiles: rows 0..7 gate features 8t.., rows 8..15 the same up features.
// h = rb(rb(g * rb(sigmoid g)) * u), g and u rounded first (src/ming_fused.zig:386-393).
struct EpiSwiGLU {
    uint16_t* h;
    int ld;
    MING_DEV void operator()(int tile, int r8, int row, float lo, float hi) const {
        const float g = rb(lo), u = rb(hi);
        const float sg = rb(1.0f / (1.0f + expf(-g)));
        h[(size_t)row * ld + tile * 8 + r8] = f2bf(rb(rb(g * sg) * u));
    }
};

constexpr int ATT_ERR_PAGES = 8;  // device error code: a K/V page copy of attn_partial_kernel never landed

struct AttnArgs {
    const uint16_t* q;  // [rows][heads*64]
    float* part;        // [rows][nsplit_max][heads][PART_STRIDE]
    KvDev kv;
    RowsDev rows;
    int layer, heads, kv_heads, nsplit_max;
    int decode = 0;  // 1: every row appends only its own position (positions before it are already cached)
    uint16_t* att = nullptr;  // when set (and at most 8 splits): the splits combine in-kernel into att [rows][heads*64]
    long long* trace = nullptr;  // launch trace: [CTA][8] globaltimer stamps (entry, wait done, keys in, .., exit at 7) or null
    // Tensor map over the page pool viewed as [pages x layers x 2 x kv_heads x
    // 16 rows][64] bf16, 16-row boxes with 128-byte swizzle (host memory; the
    // launcher passes a copy as a kernel parameter). Required.
    const CUtensorMap* tmap = nullptr;
    int* err = nullptr;  // device error word: set when a page copy never lands (bounded wait)
};

// The page pool's tensor map for attn_partial_kernel (lm.cu): false if the
// driver entry point is unavailable or rejects the shape.
bool make_kv_tensor_map(CUtensorMap* m, uint16_t* pool, long long rows);

// Step state kept on the device so one captured graph replays every decode step.
struct StepDev {
    int* seq_len;        // [max_seqs]
    int* row_seq;        // [max_batch]
    int* row_pos;        // [max_batch]
    int* step_counter;   // [2]: running counter, snapshot for this step
    uint16_t* const* out_cell;  // device cell: per-step outputs [steps][rows][H] (or null)
    float* const* stop_cell;    // device cell: [steps][rows] (or null)
};

struct FinalArgs {
    const uint16_t* x;     // residual stream [rows][H]
    const uint16_t* nw;    // final norm [H]
    const uint16_t* ws;    // stop head weight [2][H] bf16
    const uint16_t* bs;    // stop head bias [2]
    uint16_t* z;           // post-norm hidden [rows][H]
    float* stop;           // [rows]
    uint16_t* feed;        // optional copy of z as the next step's input [rows][H]
    StepDev st;
    int H, row0, advance;  // advance: bump seq_len/step counters (decode)
    float eps;
};

// Launchers (lm.cu)
cudaError_t launch_attn(const AttnArgs& a, int rows, cudaStream_t s);
bool attn_fused_combine(const AttnArgs& a);  // launch_attn wrote att itself (no combine launch needed)
cudaError_t launch_attn_combine(const float* part, RowsDev rows, int nsplit_max, int heads, uint16_t* att, int nrows,
                                cudaStream_t s);
void launch_final(const FinalArgs& a, int rows, cudaStream_t s);
void launch_step_begin(const StepDev& st, int rows, cudaStream_t s);

}  // namespace ming
