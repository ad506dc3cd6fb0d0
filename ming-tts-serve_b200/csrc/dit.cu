// dit.cu — small kernels of the flow head: attention over the few rows of one
// sequence, row assembly, the final norm/linear + CFG + Euler update.
#include <cuda_runtime.h>

#include "dit.cuh"

namespace ming {

// One warp per (row, head): scores against the L rows of the row's sequence,
// two-pass softmax, P.V, rounded (kernel A's attention tail, scale 1/8).
__global__ void dit_attention_kernel(const uint16_t* qkv, uint16_t* out, int rows, int L, int H, int heads) {
    // a programmatic dependent: q|k|v come from the previous kernel; the
    // next linear may launch and fetch its weights while this one runs
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= rows * heads) return;
    const int row = w / heads, h = w % heads, base = (row / L) * L;
    const uint16_t* q = qkv + (size_t)row * H + h * 64;
    const uint16_t* k = qkv + (size_t)rows * H;
    const uint16_t* v = qkv + (size_t)2 * rows * H;
    const float q0 = 0.125f * bf2f(q[lane]), q1 = 0.125f * bf2f(q[lane + 32]);
    float sc[16];
    float m = -INFINITY;
    for (int j = 0; j < L; j++) {
        const uint16_t* kr = k + (size_t)(base + j) * H + h * 64;
        const float s = warp_sum(q0 * bf2f(kr[lane]) + q1 * bf2f(kr[lane + 32]));
        sc[j] = s;
        m = fmaxf(m, s);
    }
    float sum = 0.f, o0 = 0.f, o1 = 0.f;
    for (int j = 0; j < L; j++) {
        const float p = expf(sc[j] - m);
        const uint16_t* vr = v + (size_t)(base + j) * H + h * 64;
        sum += p;
        o0 += p * bf2f(vr[lane]);
        o1 += p * bf2f(vr[lane + 32]);
    }
    out[(size_t)row * H + h * 64 + lane] = f2bf(o0 / sum);
    out[(size_t)row * H + h * 64 + lane + 32] = f2bf(o1 / sum);
}

void launch_dit_attention(const uint16_t* qkv, uint16_t* out, int rows, int L, int H, int heads, cudaStream_t s) {
    const int warps = rows * heads;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((warps + 3) / 4);
    cfg.blockDim = dim3(128);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, dit_attention_kernel, qkv, out, rows, L, H, heads);
}

// Rows per sequence b: [cond: t+c, hist, y | uncond: t+c0, hist, y], the
// reference's CFG batch 2 x 3 rows (kernel E, src/ming_fused.zig:247-261).
__global__ void tok_rows_kernel(const uint16_t* te, const uint16_t* ce, const uint16_t* xh, const uint16_t* xy, uint16_t* rows,
                                int B, int H) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * H) return;
    const int b = i / H, o = i % H;
    for (int half = 0; half < 2; half++) {
        uint16_t* r = rows + ((size_t)(b * 2 + half) * 3) * H;
        r[o] = f2bf(bf2f(te[o]) + bf2f(ce[((size_t)half * B + b) * H + o]));
        r[H + o] = xh[(size_t)b * H + o];
        r[2 * H + o] = xy[(size_t)b * H + o];
    }
}

void launch_tok_rows(const uint16_t* te_step, const uint16_t* ce, const uint16_t* xh, const uint16_t* xy, uint16_t* rows,
                     int B, int H, cudaStream_t s) {
    tok_rows_kernel<<<(B * H + 255) / 256, 256, 0, s>>>(te_step, ce, xh, xy, rows, B, H);
}

MING_DEV float cfg_euler(float y, float pc, float pu, float cfg, float dtv, float shift, float sqv, float sde) {
    const float f0 = rb(pc + rb(rb(pc - pu) * rb(cfg)));
    float yn = rb(y + rb(dtv * f0));
    if (shift != 0.f) yn = rb(yn + rb(rb(rb(shift) * sqv) * sde));
    return yn;
}

// One warp per (sequence, latent channel): the norm folded as in kernel F
// (w * nw dotted with x, times 1/rms), pc/pu from the last row of each half.
__global__ void tok_final_kernel(const uint16_t* x, const uint16_t* nw, const uint16_t* wf, const uint16_t* bfv, uint16_t* y,
                                 const uint16_t* sde, int step, float dtv, float sqv, float cfg, float shift, int B, int H,
                                 int latent) {
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= B * latent) return;
    const int b = w / latent, o = w % latent;
    const uint16_t* x0 = x + ((size_t)(b * 2 + 0) * 3 + 2) * H;
    const uint16_t* x1 = x + ((size_t)(b * 2 + 1) * 3 + 2) * H;
    float a0 = 0.f, a1 = 0.f, s0 = 0.f, s1 = 0.f;
    for (int k = lane; k < H; k += 32) {
        const float wv = bf2f(wf[(size_t)o * H + k]) * bf2f(nw[k]);
        const float v0 = bf2f(x0[k]), v1 = bf2f(x1[k]);
        s0 += v0 * v0;
        s1 += v1 * v1;
        a0 += wv * v0;
        a1 += wv * v1;
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    s0 = warp_sum(s0);
    s1 = warp_sum(s1);
    if (lane == 0) {
        a0 *= rsqrtf(s0 / (float)H + 1e-6f);
        a1 *= rsqrtf(s1 / (float)H + 1e-6f);
        const float pc = rb(a0 + bf2f(bfv[o])), pu = rb(a1 + bf2f(bfv[o]));
        const size_t yi = (size_t)b * latent + o;
        const float sv = sde ? bf2f(sde[((size_t)step * B + b) * latent + o]) : 0.f;
        y[yi] = f2bf(cfg_euler(bf2f(y[yi]), pc, pu, cfg, dtv, shift, sqv, sv));
    }
}

void launch_tok_final(const uint16_t* x, const uint16_t* nw, const uint16_t* wf, const uint16_t* bf, uint16_t* y,
                      const uint16_t* sde, int step, float dtv, float sqv, float cfg, float shift, int B, int H, int latent,
                      cudaStream_t s) {
    const int warps = B * latent;
    tok_final_kernel<<<(warps + 7) / 8, 256, 0, s>>>(x, nw, wf, bf, y, sde, step, dtv, sqv, cfg, shift, B, H, latent);
}

__global__ void ada_cond_kernel(const uint16_t* te, const uint16_t* ce, uint16_t* sc, int NC, int H) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= NC * H) return;
    const float c = rb(bf2f(te[i % H]) + bf2f(ce[i]));
    sc[i] = f2bf(rb(c * rb(1.0f / (1.0f + expf(-c)))));
}

void launch_ada_cond(const uint16_t* te_step, const uint16_t* ce, uint16_t* sc, int NC, int H, cudaStream_t s) {
    ada_cond_kernel<<<(NC * H + 255) / 256, 256, 0, s>>>(te_step, ce, sc, NC, H);
}

__global__ void ada_euler_kernel(const float* vel, uint16_t* y, const uint16_t* sde, int step, float dtv, float sqv, float cfg,
                                 float shift, int B, int F, int latent) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * F * latent) return;
    const float pc = rb(vel[i]), pu = rb(vel[(size_t)B * F * latent + i]);
    const float sv = sde ? bf2f(sde[(size_t)step * B * F * latent + i]) : 0.f;
    y[i] = f2bf(cfg_euler(bf2f(y[i]), pc, pu, cfg, dtv, shift, sqv, sv));
}

void launch_ada_euler(const float* vel, uint16_t* y, const uint16_t* sde, int step, float dtv, float sqv, float cfg,
                      float shift, int B, int F, int latent, cudaStream_t s) {
    ada_euler_kernel<<<(B * F * latent + 255) / 256, 256, 0, s>>>(vel, y, sde, step, dtv, sqv, cfg, shift, B, F, latent);
}

// adaLN head's latent path: out[b] = rb(mean over f of lat[b][f]) in f32,
// frames summed in order.
__global__ void latent_mean_kernel(const uint16_t* lat, uint16_t* out, int B, int F, int LAT) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * LAT) return;
    const int b = i / LAT, k = i - b * LAT;
    float s = 0.f;
    for (int f = 0; f < F; f++) s += bf2f(lat[((size_t)b * F + f) * LAT + k]);
    out[i] = f2bf(s / (float)F);
}

void launch_latent_mean(const uint16_t* lat, uint16_t* out, int B, int F, int LAT, cudaStream_t s) {
    latent_mean_kernel<<<(B * LAT + 255) / 256, 256, 0, s>>>(lat, out, B, F, LAT);
}

}  // namespace ming
