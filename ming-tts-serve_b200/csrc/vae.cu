// vae.cu — the VAE decoder (Model.vaeDecode, src/ming_model.zig:1257-1300):
// latents [T][64] -> 44.1 kHz waveform [T * 4 * 882].
//
// The reference runs the decoder's backbone in f32 (linearUpsample casts to
// f32, src/ming_model.zig:1303-1342, and MLX promotes the bf16 weights), so
// every linear here computes W x for f32 rows x with bf16 weights W: each
// linear is packed with its K doubled, [W | W], and the rows enter as two
// bf16 halves, x = hi + lo with hi = bf16(x), lo = bf16(x - hi) (about 16
// significant bits), summed in f32 on the tensor cores by the same linear
// kernels as the LM (tcgen05 at 64+ rows). The ISTFT's irfft is a linear as
// well: the DFT basis b (f32, from double) enters as hi / lo parts with K
// tripled, a_hi b_hi + a_hi b_lo + a_lo b_hi. Attention is causal over a
// sliding window of vae_window positions (slidingMask, :617-635).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "dispatch.cuh"

using namespace ming;
using namespace ming::rt;

namespace ming {
namespace vaek {  // the decoder's constants, prologues, epilogues and kernels

constexpr int VAE_PATCH = 4;              // latents are upsampled x4 (VAE_PATCH)
constexpr int HOP = 882;                  // ISTFT hop
constexpr int NFFT = 3528;                // ISTFT size (4 hops)
constexpr int NBIN = NFFT / 2 + 1;        // 1765 bins
constexpr int HEAD_OUT = 2 * NBIN;        // head features: log-magnitudes, phases
constexpr int DFT_K = 3 * HEAD_OUT;       // hi | hi | lo sections of the spectrum
constexpr int DFT_KP = (DFT_K + 63) / 64 * 64;
constexpr int DFT_ROWS = (NFFT + 127) / 128 * 128;  // whole 128-feature blocks for the tcgen05 linear

// ---- prologues: f32 rows as bf16 parts over K sections ----

// Section s of width Kp holds bf16(v) (hi) or bf16(v - bf16(v)) (lo) of
// v = x[row][k - s Kp], as bit s of lo_mask says; k beyond the sections is 0.
struct ProSplitF32 {
    const float* x;
    int ld, Kp, nsec, lo_mask;
    int r0;
    MING_DEV void init(int r0_, int, float*) { r0 = r0_; }
    MING_DEV float y(int row, int k) const {
        const int s = k / Kp;
        if (s >= nsec) return 0.f;
        const float v = x[(size_t)(r0 + row) * ld + (k - s * Kp)];
        const float hi = rb(v);
        return (lo_mask >> s) & 1 ? rb(v - hi) : hi;
    }
    MING_DEV float post(int) const { return 1.f; }
};

// MLX fast_rms_norm on an f32 row (x rsqrt(mean(x^2) + eps) w, in f32), then
// split into [hi | lo] over 2K
struct ProRmsSplitF32 {
    const float* x;
    const uint16_t* nw;
    int ld, K;
    float eps;
    int r0;
    float* inv;
    MING_DEV void init(int r0_, int nrows, float* aux) {
        r0 = r0_;
        inv = aux;
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int r = warp; r < nrows; r += LIN_WARPS) {
            const float* xr = x + (size_t)(r0 + r) * ld;
            float s = 0.f;
            for (int k = lane; k < K; k += 32) s += xr[k] * xr[k];
            s = warp_sum(s);
            if (lane == 0) aux[r] = rsqrtf(s / (float)K + eps);
        }
    }
    MING_DEV float y(int row, int k) const {
        const int kk = k < K ? k : k - K;
        const float v = x[(size_t)(r0 + row) * ld + kk] * inv[row] * bf2f(nw[kk]);
        const float hi = rb(v);
        return k < K ? hi : rb(v - hi);
    }
    MING_DEV float post(int) const { return 1.f; }
};

// ---- epilogues (f32 outputs) ----

// q|k|v in the LM's tile order (tile t of a block: head t/4, dims d0 = 8 (t%4)
// .. +7 and their RoPE partners d0 + 32 ..): bias, then RoPE at position =
// row (MLX fast_rope, non-traditional, angle pos 2^(-(d/32) log2 theta)) in
// f32 without rounding
struct EpiQKVf32 {
    const float* bias;
    float *q, *k, *v;
    int heads, kv_heads;
    float log2_theta;
    MING_DEV void operator()(int tile, int r8, int row, float lo, float hi) const {
        const int qt = heads * 4, kt = kv_heads * 4;
        const int which = tile < qt ? 0 : (tile < qt + kt ? 1 : 2);
        const int lt = which == 0 ? tile : (which == 1 ? tile - qt : tile - qt - kt);
        const int h = lt >> 2, d = (lt & 3) * 8 + r8;
        float x1 = lo + bias[tile * 16 + r8];
        float x2 = hi + bias[tile * 16 + r8 + 8];
        if (which < 2) {
            const float th = (float)row * exp2f(-((float)d / 32.0f) * log2_theta);
            float sn, cs;
            sincosf(th, &sn, &cs);
            const float a = x1 * cs - x2 * sn, b = x1 * sn + x2 * cs;
            x1 = a;
            x2 = b;
        }
        float* dst = which == 0 ? q + ((size_t)row * heads + h) * HD
                                : (which == 1 ? k : v) + ((size_t)row * kv_heads + h) * HD;
        dst[d] = x1;
        dst[d + 32] = x2;
    }
};

// out = res + W x (o_proj, down: no bias); out may alias res
struct EpiResidualF32 {
    const float* res;
    float* out;
    int ld;
    MING_DEV void operator()(int tile, int r8, int row, float lo, float hi) const {
        const size_t i0 = (size_t)row * ld + tile * 16 + r8, i1 = i0 + 8;
        const float x0 = res[i0], x1 = res[i1];
        out[i0] = x0 + lo;
        out[i1] = x1 + hi;
    }
};

// gate|up tiles (rows 0..7 gate, 8..15 up of features 8t..): silu(g) u in f32
struct EpiSwiGLUf32 {
    float* h;
    int ld;
    MING_DEV void operator()(int tile, int r8, int row, float lo, float hi) const {
        const float sg = 1.0f / (1.0f + expf(-lo));
        h[(size_t)row * ld + tile * 8 + r8] = (lo * sg) * hi;
    }
};

// ---- kernels ----

// Decoder._linear_upsample_1d (align_corners false) in f32: output row i at
// source position p = (i + 0.5) / 4 - 0.5 mixes rows floor(p), floor(p) + 1
// (clamped) with weights 1 - w, w, w = p - floor(p): lv (1 - w) + rv w, each
// product rounded before the sum as the reference's graph does.
__global__ void vae_upsample_kernel(const uint16_t* x, int T, int H, float* out) {
    const int i = blockIdx.x;
    const float p = __fsub_rn(__fdiv_rn(__fadd_rn((float)i, 0.5f), (float)VAE_PATCH), 0.5f);
    const float lf = floorf(p);
    const int l = (int)lf;
    const float w = __fsub_rn(p, lf), wl = __fsub_rn(1.0f, w);
    const int a = min(max(l, 0), T - 1), b = min(max(l + 1, 0), T - 1);
    for (int f = threadIdx.x; f < H; f += blockDim.x)
        out[(size_t)i * H + f] = __fadd_rn(__fmul_rn(bf2f(x[(size_t)a * H + f]), wl), __fmul_rn(bf2f(x[(size_t)b * H + f]), w));
}

// Causal sliding-window attention in f32 (slidingMask: key kp visible from
// query qp when qp - window < kp <= qp; SDPA with scale 1/8). A CTA takes
// VA_RB consecutive query rows and one kv head: it stages the keys and values
// of the rows' windows (at most window - 1 + VA_RB positions) and the q rows
// of its (row, query head) pairs in shared memory once, then warp w runs the
// pairs w, w + 8, ...: a lane per two keys for the scores (window <= 64,
// checked at set-up), then a lane per two dims for P.V, four keys' loads in
// flight at a time and their probabilities read from shared memory at once.
// Staging once per block instead of reading every (row, head)'s window from
// global memory cuts the L2 traffic ~30x; the arithmetic of each (row, head),
// summation order included, is unchanged.
constexpr int VA_RB = 4;                 // query rows per CTA
constexpr int VA_WARPS = 8;
constexpr int VA_KS = HD + 4;            // row stride (floats) of the staged K/V: the float4 reads of
                                         // 8 lanes on consecutive rows fall on distinct bank groups
constexpr int VA_MAXK = 64 - 1 + VA_RB;  // positions of a block's windows
constexpr int VA_MAXG = 8;               // query heads per kv head staged (the context's limit, checked at set-up)
__global__ void __launch_bounds__(VA_WARPS * 32) vae_attention_kernel(const float* q, const float* k, const float* v,
                                                                      float* o, int F, int heads, int kvh, int window,
                                                                      float scale) {
    __shared__ __align__(16) float sK[VA_MAXK * VA_KS];
    __shared__ __align__(16) float sV[VA_MAXK * VA_KS];
    __shared__ __align__(16) float sQ[VA_RB * VA_MAXG * HD];
    __shared__ __align__(16) float sP[VA_WARPS][64];  // each warp's probabilities of its current pair
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * VA_RB, g = blockIdx.y, grp = heads / kvh;
    const int k0 = max(0, r0 - window + 1), nk = min(F, r0 + VA_RB) - k0;  // nk <= VA_MAXK
    const int nr = min(VA_RB, F - r0), np = nr * grp;                      // rows and (row, head) pairs
    for (int e = threadIdx.x; e < nk * (HD / 4); e += blockDim.x) {
        const int j = e / (HD / 4), c4 = e % (HD / 4);
        const size_t src = ((size_t)(k0 + j) * kvh + g) * HD + 4 * c4;
        *reinterpret_cast<float4*>(sK + j * VA_KS + 4 * c4) = *reinterpret_cast<const float4*>(k + src);
        *reinterpret_cast<float4*>(sV + j * VA_KS + 4 * c4) = *reinterpret_cast<const float4*>(v + src);
    }
    for (int e = threadIdx.x; e < np * (HD / 4); e += blockDim.x) {
        const int pr = e / (HD / 4), c4 = e % (HD / 4), row = r0 + pr / grp, h = g * grp + pr % grp;
        *reinterpret_cast<float4*>(sQ + pr * HD + 4 * c4) =
            *reinterpret_cast<const float4*>(q + ((size_t)row * heads + h) * HD + 4 * c4);
    }
    __syncthreads();
    for (int pr = warp; pr < np; pr += VA_WARPS) {  // warp-uniform
        const int row = r0 + pr / grp, h = g * grp + pr % grp;
        const int j0 = max(0, row - window + 1), n = row - j0 + 1;  // keys j0 .. row, n <= window
        const float* kb = sK + (j0 - k0) * VA_KS;
        const float* vb = sV + (j0 - k0) * VA_KS;
        const float* qs = sQ + pr * HD;
        // the lane's keys j = lane and lane + 32 over the dims in order, one q
        // load per step for both
        const bool u0 = lane < n, u1 = lane + 32 < n;
        const float* kr0 = kb + lane * VA_KS;
        const float* kr1 = kb + (lane + 32) * VA_KS;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
        for (int d4 = 0; d4 < HD / 4; d4++) {
            const float4 qq = *reinterpret_cast<const float4*>(qs + 4 * d4);
            if (u0) {
                const float4 kk = *reinterpret_cast<const float4*>(kr0 + 4 * d4);
                a0 += qq.x * kk.x;
                a0 += qq.y * kk.y;
                a0 += qq.z * kk.z;
                a0 += qq.w * kk.w;
            }
            if (u1) {
                const float4 kk = *reinterpret_cast<const float4*>(kr1 + 4 * d4);
                a1 += qq.x * kk.x;
                a1 += qq.y * kk.y;
                a1 += qq.z * kk.z;
                a1 += qq.w * kk.w;
            }
        }
        const float s0 = u0 ? a0 * scale : -INFINITY, s1 = u1 ? a1 * scale : -INFINITY;
        const float m = warp_max(fmaxf(s0, s1));
        const float p0 = u0 ? expf(s0 - m) : 0.f, p1 = u1 ? expf(s1 - m) : 0.f;
        const float L = warp_sum(p0 + p1);
        // P.V over the keys in order, the probabilities read four at a time
        // from the warp's row of sP
        float* pw = sP[warp];
        pw[lane] = p0;
        pw[lane + 32] = p1;
        __syncwarp();
        float2 acc = make_float2(0.f, 0.f);
        int j = 0;
        for (; j + 4 <= n; j += 4) {  // n is warp-uniform
            const float4 p4 = *reinterpret_cast<const float4*>(pw + j);
            const float pj[4] = {p4.x, p4.y, p4.z, p4.w};
            float2 vv[4];
#pragma unroll
            for (int u = 0; u < 4; u++) vv[u] = *reinterpret_cast<const float2*>(vb + (j + u) * VA_KS + 2 * lane);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                acc.x += pj[u] * vv[u].x;
                acc.y += pj[u] * vv[u].y;
            }
        }
        for (; j < n; j++) {
            const float pj = pw[j];
            const float2 vv = *reinterpret_cast<const float2*>(vb + j * VA_KS + 2 * lane);
            acc.x += pj * vv.x;
            acc.y += pj * vv.y;
        }
        __syncwarp();  // every lane read pw before the next pair overwrites it
        float* orow = o + ((size_t)row * heads + h) * HD;
        orow[2 * lane] = acc.x / L;
        orow[2 * lane + 1] = acc.y / L;
    }
}

// The ISTFT's spectrum from the head's output p [F][3530]: magnitude
// min(exp(p[j]), 100), phase p[1765 + j], as (re | im) [F][3530] in f32.
__global__ void vae_spectrum_kernel(const float* p, float* spec, int F) {
    const int f = blockIdx.x;
    for (int j = threadIdx.x; j < NBIN; j += blockDim.x) {
        const float mag = fminf(expf(p[(size_t)f * HEAD_OUT + j]), 100.0f);
        float sn, cs;
        sincosf(p[(size_t)f * HEAD_OUT + NBIN + j], &sn, &cs);
        spec[(size_t)f * HEAD_OUT + j] = mag * cs;
        spec[(size_t)f * HEAD_OUT + NBIN + j] = mag * sn;
    }
}

// Windowed overlap-add at hop 882 (n_fft = 4 hops), divided by the window
// envelope, with the "same" trim: output sample i is position o = i + 1323 of
// the (F + 3) hop blocks. Frame parts are added in the reference's order
// (part 3 of frame b - 3 first, part 0 of frame b last; missing frames add
// zero), the envelope in frame order.
__global__ void vae_ola_kernel(const float* frames, const float* win, int F, float* wave) {
    const int n_out = F * HOP;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_out) return;
    const int o = i + (NFFT - HOP) / 2, b = o / HOP, kk = o - b * HOP;
    float acc = 0.f, env = 0.f;
#pragma unroll
    for (int j = 3; j >= 0; j--) {
        const int t = b - j;  // frame whose part j covers block b
        if (t < 0 || t >= F) continue;
        const float w = win[j * HOP + kk];
        acc = __fadd_rn(acc, __fmul_rn(frames[(size_t)t * NFFT + j * HOP + kk], w));
        env = __fadd_rn(env, __fmul_rn(w, w));
    }
    wave[i] = __fdiv_rn(acc, fmaxf(env, 1e-11f));
}

}  // namespace vaek
}  // namespace ming

using namespace ming::vaek;

namespace ming {
namespace rt {

// A bf16 linear [out][K] repacked with its K doubled ([W | W]) in the given
// row order; `in` must be K.
static int pack_doubled(ming_ctx* c, const std::string& prefix, bool bias, const std::vector<std::string>& extra,
                 const std::vector<RowRef>& rows, PackedLin& pl, int* out_dim = nullptr) {
    std::vector<std::string> names{prefix};
    names.insert(names.end(), extra.begin(), extra.end());
    std::vector<LinearSrc> srcs(names.size());
    std::vector<std::vector<uint16_t>> wide(names.size());
    std::vector<std::string> wnames;
    for (size_t i = 0; i < names.size(); i++) {
        int rc = lin_src(c, names[i], srcs[i], bias);
        if (rc) return rc;
        if (srcs[i].fmt != 16) return fail(MING_ERR_INVALID, names[i] + ": the VAE decoder takes bf16 weights");
        const int O = srcs[i].out, K = srcs[i].in;
        wide[i].resize((size_t)O * 2 * K);
        for (int r = 0; r < O; r++) {
            std::memcpy(&wide[i][(size_t)r * 2 * K], srcs[i].w + (size_t)r * K, (size_t)K * 2);
            std::memcpy(&wide[i][(size_t)r * 2 * K + K], srcs[i].w + (size_t)r * K, (size_t)K * 2);
        }
        srcs[i].w = wide[i].data();
        srcs[i].in = 2 * K;
        wnames.push_back(names[i] + ".weight");
    }
    if (out_dim) *out_dim = srcs[0].out;
    return upload_packed(c, srcs, wnames, rows, pl);
}

// Plain row order padded with zero rows to `multiple` rows (128: whole
// feature blocks of the tcgen05 linear).
static std::vector<RowRef> plain_rows(int out, int multiple = 16) {
    std::vector<RowRef> rows(((out + multiple - 1) / multiple) * multiple);
    for (size_t i = 0; i < rows.size(); i++) rows[i] = (int)i < out ? RowRef{0, (int)i} : RowRef{-1, 0};
    return rows;
}

static uint16_t bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static float bf16_val(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

int vae_finalize(ming_ctx* c) {
    const ming_cfg& f = c->cfg;
    if (f.vae_ff < 64 || f.vae_ff % 64 || f.vae_window < 1 || f.vae_window > 64 || f.vae_max_latents < 1)
        return fail(MING_ERR_INVALID,
                    "bad VAE decoder shape (vae_ff a multiple of 64, vae_window 1..64, vae_max_latents >= 1)");
    if (f.kv_heads < 1 || f.heads % f.kv_heads || f.heads / f.kv_heads > VA_MAXG)
        return fail(MING_ERR_INVALID, "VAE attention: heads must be a multiple of kv_heads, at most 8 per kv head");
    const int H = f.hidden, QD = f.heads * HD, KD = f.kv_heads * HD, FF = f.vae_ff;
    const std::string D = "audio.decoder";
    int rc, od = 0;
    if ((rc = ::ming::rt::pack_plain(c, D + ".fc1", true, c->vae_fc1, &od))) return rc;
    if (od != H || c->vae_fc1.w.K != 64) return fail(MING_ERR_INVALID, D + ".fc1 must be [hidden, 64]");
    c->vae.resize(f.vae_layers);
    for (int l = 0; l < f.vae_layers; l++) {
        const std::string p = D + ".decoder.layers." + std::to_string(l);
        auto& L = c->vae[l];
        LinearSrc q, k, v, o, g, u, d;
        if ((rc = lin_src(c, p + ".self_attn.q_proj", q, true)) || (rc = lin_src(c, p + ".self_attn.k_proj", k, true)) ||
            (rc = lin_src(c, p + ".self_attn.v_proj", v, true)) || (rc = lin_src(c, p + ".self_attn.o_proj", o, false)) ||
            (rc = lin_src(c, p + ".mlp.gate_proj", g, false)) || (rc = lin_src(c, p + ".mlp.up_proj", u, false)) ||
            (rc = lin_src(c, p + ".mlp.down_proj", d, false)))
            return rc;
        if (q.out != QD || k.out != KD || v.out != KD || q.in != H || o.out != H || o.in != QD || g.out != FF || u.out != FF ||
            d.out != H || d.in != FF)
            return fail(MING_ERR_INVALID, p + ": decoder linear shapes do not match hidden / heads / vae_ff");
        // q|k|v: the LM's rope-half tiles; gate|up: 8 gate rows then the same 8 up rows
        std::vector<RowRef> rows;
        const int nh[3] = {f.heads, f.kv_heads, f.kv_heads};
        for (int b = 0; b < 3; b++)
            for (int t = 0; t < nh[b] * 4; t++)
                for (int r = 0; r < 16; r++) {
                    const int h = t / 4, d0 = (t % 4) * 8;
                    rows.push_back({b, h * 64 + (r < 8 ? d0 + r : 32 + d0 + r - 8)});
                }
        if ((rc = pack_doubled(c, p + ".self_attn.q_proj", true, {p + ".self_attn.k_proj", p + ".self_attn.v_proj"}, rows,
                               L.qkv)))
            return rc;
        if ((rc = pack_doubled(c, p + ".self_attn.o_proj", false, {}, plain_rows(H), L.o))) return rc;
        if ((rc = pack_doubled(c, p + ".mlp.down_proj", false, {}, plain_rows(H), L.down))) return rc;
        rows.clear();
        for (int t = 0; t < FF / 8; t++)
            for (int r = 0; r < 16; r++) rows.push_back({r < 8 ? 0 : 1, t * 8 + (r & 7)});
        if ((rc = pack_doubled(c, p + ".mlp.gate_proj", false, {p + ".mlp.up_proj"}, rows, L.gu))) return rc;
        if ((rc = upload_raw(c, p + ".input_layernorm.weight", MING_DTYPE_BF16, H, (void**)&L.ln1))) return rc;
        if ((rc = upload_raw(c, p + ".post_attention_layernorm.weight", MING_DTYPE_BF16, H, (void**)&L.ln2))) return rc;
    }
    if ((rc = upload_raw(c, D + ".decoder.norm.weight", MING_DTYPE_BF16, H, (void**)&c->vae_norm))) return rc;
    if ((rc = pack_doubled(c, D + ".head.out", true, {}, plain_rows(HEAD_OUT, 128), c->vae_head, &od))) return rc;
    if (od != HEAD_OUT) return fail(MING_ERR_INVALID, D + ".head.out must have 3530 outputs (2 x 1765 bins)");
    if ((rc = upload_raw(c, D + ".head.istft.window", MING_DTYPE_F32, NFFT, (void**)&c->vae_win))) return rc;
    {
        // irfft (n 3528, "backward" norm) as a linear over the spectrum
        // (re | im) [3530]: frame[n] = sum_j c_j (re_j cos(2 pi j n / N) -
        // im_j sin(2 pi j n / N)) / N, c = 1 for the DC and Nyquist bins
        // (whose imaginary parts irfft ignores) and 2 otherwise. The f32
        // basis (from double) enters as hi | lo | hi against the spectrum's
        // hi | hi | lo sections; rows past 3528 and K past 3 x 3530 are zero.
        std::vector<uint16_t> basis((size_t)DFT_ROWS * DFT_KP, 0);
        for (int n = 0; n < NFFT; n++) {
            uint16_t* row = &basis[(size_t)n * DFT_KP];
            for (int j = 0; j < HEAD_OUT; j++) {
                const int bin = j < NBIN ? j : j - NBIN;
                const bool imag = j >= NBIN;
                const double cj = (bin == 0 || bin == NFFT / 2) ? 1.0 : 2.0;
                const long long m = ((long long)bin * n) % NFFT;
                const double ang = 2.0 * 3.14159265358979323846 * (double)m / (double)NFFT;
                double b = imag ? -std::sin(ang) : std::cos(ang);
                if (imag && (bin == 0 || bin == NFFT / 2)) b = 0.0;
                const float bf = (float)(cj * b / (double)NFFT);
                const uint16_t hi = bf16_bits(bf), lo = bf16_bits(bf - bf16_val(hi));
                row[j] = hi;
                row[HEAD_OUT + j] = lo;
                row[2 * HEAD_OUT + j] = hi;
            }
        }
        LinearSrc s{};
        s.fmt = 16;
        s.out = DFT_ROWS;
        s.in = DFT_KP;
        s.w = basis.data();
        std::vector<RowRef> rows(DFT_ROWS);
        for (int i = 0; i < DFT_ROWS; i++) rows[i] = RowRef{0, i};
        if ((rc = upload_packed(c, {s}, {"istft.dft_basis"}, rows, c->vae_dft))) return rc;
    }
    const size_t R = (size_t)VAE_PATCH * f.vae_max_latents;
    rc = MING_OK;
    c->v_lat = c->mem.alloc<uint16_t>((size_t)f.vae_max_latents * 64, &rc);
    c->v_fc1 = c->mem.alloc<uint16_t>((size_t)f.vae_max_latents * H, &rc);
    c->v_x = c->mem.alloc<float>(R * H, &rc);
    c->v_q = c->mem.alloc<float>(R * QD, &rc);
    c->v_k = c->mem.alloc<float>(R * KD, &rc);
    c->v_v = c->mem.alloc<float>(R * KD, &rc);
    c->v_att = c->mem.alloc<float>(R * QD, &rc);
    c->v_h = c->mem.alloc<float>(R * FF, &rc);
    c->v_head = c->mem.alloc<float>(R * HEAD_OUT, &rc);
    c->v_spec = c->mem.alloc<float>(R * HEAD_OUT, &rc);
    c->v_frames = c->mem.alloc<float>(R * NFFT, &rc);
    c->v_wave = c->mem.alloc<float>(R * HOP, &rc);
    return rc;
}

}  // namespace rt
}  // namespace ming

extern "C" int ming_cuda_vae_decode(ming_ctx* c, const uint16_t* latents, int T, float* wave, int kind) {
    if (!c || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    const ming_cfg& f = c->cfg;
    if (f.vae_layers < 1) return fail(MING_ERR_INVALID, "no VAE decoder configured");
    if (!latents || !wave || T < 1) return fail(MING_ERR_INVALID, "bad argument");
    if (T > f.vae_max_latents) return fail(MING_ERR_INVALID, "more latents than vae_max_latents");
    CK(cudaSetDevice(c->device));
    cudaStream_t s = c->stream;
    const int H = f.hidden, F = VAE_PATCH * T, QD = f.heads * HD, KD = f.kv_heads * HD;
    CK(cudaMemcpyAsync(c->v_lat, latents, (size_t)T * 64 * 2,
                       kind == MING_PTR_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
    // fc1 in bf16 (the latents' dtype), then the upsample to f32
    run_linear(c, c->vae_fc1.w, ProPlain{c->v_lat, 64, 0}, EpiAct{c->v_fc1, nullptr, c->vae_fc1.w.bias, H, 0, H}, T, s);
    vae_upsample_kernel<<<F, 256, 0, s>>>(c->v_fc1, T, H, c->v_x);
    const float log2_theta = log2f(f.rope_theta);
    for (auto& L : c->vae) {
        run_linear(c, L.qkv.w, ProRmsSplitF32{c->v_x, L.ln1, H, H, f.rms_eps, 0, nullptr},
                   EpiQKVf32{L.qkv.w.bias, c->v_q, c->v_k, c->v_v, f.heads, f.kv_heads, log2_theta}, F, s);
        vae_attention_kernel<<<dim3((F + VA_RB - 1) / VA_RB, f.kv_heads), VA_WARPS * 32, 0, s>>>(
            c->v_q, c->v_k, c->v_v, c->v_att, F, f.heads, f.kv_heads, f.vae_window, 0.125f);
        run_linear(c, L.o.w, ProSplitF32{c->v_att, QD, QD, 2, 2, 0}, EpiResidualF32{c->v_x, c->v_x, H}, F, s);
        run_linear(c, L.gu.w, ProRmsSplitF32{c->v_x, L.ln2, H, H, f.rms_eps, 0, nullptr}, EpiSwiGLUf32{c->v_h, f.vae_ff}, F,
                   s);
        run_linear(c, L.down.w, ProSplitF32{c->v_h, f.vae_ff, f.vae_ff, 2, 2, 0}, EpiResidualF32{c->v_x, c->v_x, H}, F, s);
    }
    // final norm folded into the head's prologue; then the ISTFT
    run_linear(c, c->vae_head.w, ProRmsSplitF32{c->v_x, c->vae_norm, H, H, f.rms_eps, 0, nullptr},
               EpiAct{nullptr, c->v_head, c->vae_head.w.bias, HEAD_OUT, 3, HEAD_OUT}, F, s);
    vae_spectrum_kernel<<<F, 256, 0, s>>>(c->v_head, c->v_spec, F);
    run_linear(c, c->vae_dft.w, ProSplitF32{c->v_spec, HEAD_OUT, HEAD_OUT, 3, 4, 0},
               EpiAct{nullptr, c->v_frames, nullptr, NFFT, 3, NFFT}, F, s);
    vae_ola_kernel<<<(F * HOP + 255) / 256, 256, 0, s>>>(c->v_frames, c->vae_win, F, c->v_wave);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(wave, c->v_wave, (size_t)F * HOP * 4,
                       kind == MING_PTR_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s));
    if (kind == MING_PTR_HOST) CK(cudaStreamSynchronize(s));
    (void)KD;
    return MING_OK;
}
