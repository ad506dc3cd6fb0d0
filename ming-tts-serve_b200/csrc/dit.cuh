// dit.cuh — the per-step DiT flow head on the tiled linear kernel.
//
// Token mode is the reference's head (src/ming_model.zig:770-797,1159-1215;
// fused kernels A-F, src/ming_fused.zig:144-289): rows [t+c, x_emb(hist),
// x_emb(y)] per CFG half, RMSNorm blocks, interleaved rotary.
// adaLN mode is the benchmark's adaLN-Zero head (6 blocks x 768, a 4 x 64
// latent patch, no reference code): frames of the latent patch as rows,
// LayerNorm + (shift, scale, gate) modulation from SiLU(c), same rotary,
// attention, gelu MLP and Euler/CFG update.
#pragma once

#include "linear.cuh"

namespace ming {

// q|k|v tiles with neighbour interleave: tile row r (<8) -> feature
// 16*lt + 2r, row r+8 -> 16*lt + 2r + 1 of block b = tile / (H/16).
// Rotary pairs (2i, 2i+1) at position row % L, rounded once (kernel A).
struct EpiDitQKV {
    const float* bias;
    uint16_t* qkv;  // [3][rows][H]
    const float* inv_freq;  // [32]
    int H, L, rows;
    MING_DEV void operator()(int tile, int r8, int row, float lo, float hi) const {
        const int tpb = H / 16, b = tile / tpb, lt = tile % tpb;
        const int f = lt * 16 + 2 * r8;
        float e = rb(lo + bias[tile * 16 + r8]);
        float o = rb(hi + bias[tile * 16 + r8 + 8]);
        if (b < 2) {
            const int i = (f % 64) / 2, pos = row % L;
            const float ang = (float)pos * inv_freq[i];
            float s, c;
            sincosf(ang, &s, &c);
            const float ne = e * c - o * s, no = e * s + o * c;
            e = ne;
            o = no;
        }
        uint16_t* dst = qkv + ((size_t)b * rows + row) * H + f;
        dst[0] = f2bf(e);
        dst[1] = f2bf(o);
    }
};

// adaLN gated residual: out = rb(x + rb(gate * rb(v + bias))), gate from the
// row's condition (rows_per_cond consecutive rows share one).
struct EpiGatedRes {
    const uint16_t* res;
    uint16_t* out;
    const float* bias;
    const uint16_t* gate;  // [cond rows][mod_ld]
    int ld, mod_ld, rows_per_cond;
    MING_DEV void operator()(int tile, int r8, int row, float lo, float hi) const {
        const int c = row / rows_per_cond;
        const int f0 = tile * 16 + r8, f1 = f0 + 8;
        const size_t i0 = (size_t)row * ld + f0, i1 = (size_t)row * ld + f1;
        // every load before the first store: out may alias res, so a load after
        // a store would wait for it
        const float g0 = bf2f(gate[(size_t)c * mod_ld + f0]), g1 = bf2f(gate[(size_t)c * mod_ld + f1]);
        const float x0 = bf2f(res[i0]), x1 = bf2f(res[i1]);
        const float b0 = bias ? bias[f0] : 0.f, b1 = bias ? bias[f1] : 0.f;
        out[i0] = f2bf(x0 + rb(g0 * rb(lo + b0)));
        out[i1] = f2bf(x1 + rb(g1 * rb(hi + b1)));
    }
};

// Token rows of the adaLN head: row (half h, batch b, frame f) -> latent of b.
struct ProLatent {
    const uint16_t* lat;  // [B][F][latent]
    int B, F, latent;
    int r0;
    MING_DEV void init(int r0_, int, float*) { r0 = r0_; }
    MING_DEV float y_at(int ar, int k) const {
        const int f = ar % F, b = (ar / F) % B;
        return bf2f(lat[((size_t)b * F + f) * latent + k]);
    }
    MING_DEV float y(int row, int k) const { return y_at(r0 + row, k); }
    MING_DEV float post(int) const { return 1.f; }
};

// Launchers (dit.cu)
void launch_dit_attention(const uint16_t* qkv, uint16_t* out, int rows, int L, int H, int heads, cudaStream_t s);
// Token head: assemble the 6 rows per sequence [t+c, hist, y] (kernel E).
void launch_tok_rows(const uint16_t* te_step, const uint16_t* ce, const uint16_t* xh, const uint16_t* xy, uint16_t* rows,
                     int B, int H, cudaStream_t s);
// Token head final (kernel F): RMSNorm + linear on the last row of each half,
// CFG combine and Euler step, per sequence.
void launch_tok_final(const uint16_t* x, const uint16_t* nw, const uint16_t* wf, const uint16_t* bf, uint16_t* y,
                      const uint16_t* sde, int step, float dtv, float sqv, float cfg, float shift, int B, int H, int latent,
                      cudaStream_t s);
// adaLN: c = rb(te + ce); sc = silu chain. [2B][H]
void launch_ada_cond(const uint16_t* te_step, const uint16_t* ce, uint16_t* sc, int NC, int H, cudaStream_t s);
// adaLN latent path: out [B][latent] = rb(mean over the F frames of lat [B][F][latent]).
void launch_latent_mean(const uint16_t* lat, uint16_t* out, int B, int F, int LAT, cudaStream_t s);
// CFG + Euler on velocities vel [2B*F][latent] (f32 unrounded linear outputs).
void launch_ada_euler(const float* vel, uint16_t* y, const uint16_t* sde, int step, float dtv, float sqv, float cfg,
                      float shift, int B, int F, int latent, cudaStream_t s);

}  // namespace ming
