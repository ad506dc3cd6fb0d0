// lm.cu — paged split-K decode attention, final norm + stop head, step
// bookkeeping kernels.
#include <cuda_runtime.h>

#include "lm.cuh"

namespace ming {

// One CTA per (split, kv head, row). Scores of the 7 query heads sharing the kv
// head against the split's positions (two-pass softmax inside the split, as
// the reference's LB kernel, src/ming_fused.zig:326-374), then P.V.
// Partial (m, l, acc) go to `part` for the O prologue to combine.
__global__ void __launch_bounds__(128) attn_partial_kernel(AttnArgs a) {
    constexpr int MAXG = 8;  // query heads per kv head (<= 8)
    __shared__ float sq[MAXG][HD];
    __shared__ uint32_t sk[PAGE][HD / 2 + 1];  // padded: 16 rows on distinct banks
    __shared__ uint16_t sv[PAGE][HD];
    __shared__ float sc[MAXG][ATT_SPLIT];
    __shared__ float sm[MAXG], sl[MAXG];
    const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = a.heads / a.kv_heads;
    const int pos = a.rows.pos[row], seq = a.rows.seq[row];
    const int n = pos + 1, p0 = split * ATT_SPLIT, p1 = min(n, p0 + ATT_SPLIT);
    float* out = a.part + ((size_t)row * a.nsplit_max + split) * a.heads * PART_STRIDE;
    if (p0 >= n) return;  // split unused for this row (never read by the combine)
    for (int e = tid; e < grp * HD; e += 128) {
        const int i = e / HD, d = e % HD;
        sq[i][d] = 0.125f * bf2f(a.q[(size_t)row * a.heads * HD + (kh * grp + i) * HD + d]);
    }
    const int* bt = a.kv.bt + (size_t)seq * a.kv.bt_ld;
    // pass 1: scores
    for (int pb = p0; pb < p1; pb += PAGE) {
        const int page = bt[pb / PAGE];
        const uint16_t* kp = a.kv.pool + kv_index(a.kv, page, a.layer, 0, kh, 0);
        __syncthreads();
        {
            const int slot = tid >> 3, c = (tid & 7) * 8;  // 128 threads x 8 dims
            const uint4 v = *reinterpret_cast<const uint4*>(kp + slot * HD + c);
            sk[slot][c / 2] = v.x;
            sk[slot][c / 2 + 1] = v.y;
            sk[slot][c / 2 + 2] = v.z;
            sk[slot][c / 2 + 3] = v.w;
        }
        __syncthreads();
        if (tid < grp * PAGE) {
            const int i = tid / PAGE, slot = tid % PAGE, p = pb + slot;
            if (p < p1) {
                float s = 0.f;
#pragma unroll 8
                for (int d2 = 0; d2 < HD / 2; d2++) {
                    const float2 kv2 = unpack_bf16x2(sk[slot][d2]);
                    s += sq[i][2 * d2] * kv2.x + sq[i][2 * d2 + 1] * kv2.y;
                }
                sc[i][p - p0] = s;
            }
        }
    }
    __syncthreads();
    const int len = p1 - p0;
    for (int i = warp; i < grp; i += 4) {
        float m = -INFINITY;
        for (int j = lane; j < len; j += 32) m = fmaxf(m, sc[i][j]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < len; j += 32) {
            const float p = expf(sc[i][j] - m);
            sc[i][j] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) { sm[i] = m; sl[i] = l; }
    }
    // pass 2: P.V; thread owns dim d for heads i0, i0+2, i0+4, i0+6
    const int d = tid & 63, i0 = tid >> 6;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int pb = p0; pb < p1; pb += PAGE) {
        const int page = bt[pb / PAGE];
        const uint16_t* vp = a.kv.pool + kv_index(a.kv, page, a.layer, 1, kh, 0);
        __syncthreads();
        reinterpret_cast<uint4*>(&sv[0][0])[tid] = reinterpret_cast<const uint4*>(vp)[tid];
        __syncthreads();
        const int cnt = min(PAGE, p1 - pb);
        for (int j = 0; j < cnt; j++) {
            const float v = bf2f(sv[j][d]);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = i0 + 2 * u;
                if (i < grp) acc[u] += sc[i][pb - p0 + j] * v;
            }
        }
    }
    for (int u = 0; u < 4; u++) {
        const int i = i0 + 2 * u;
        if (i >= grp) continue;
        float* o = out + (size_t)(kh * grp + i) * PART_STRIDE;
        o[2 + d] = acc[u];
        if (d == 0) { o[0] = sm[i]; o[1] = sl[i]; }
    }
}

void launch_attn(const AttnArgs& a, int rows, cudaStream_t s) {
    dim3 grid(a.nsplit_max, a.kv_heads, rows);
    attn_partial_kernel<<<grid, 128, 0, s>>>(a);
}

// Final RMSNorm (MLX fast_rms_norm: rb(w * rb(x * inv))) and the stop head:
// p = softmax(f32(rb(z Ws^T + b)))[1] (src/ming_model.zig:1033-1038).
__global__ void __launch_bounds__(256) final_kernel(FinalArgs a) {
    const int row = a.row0 + blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ float red[3][8];
    const uint16_t* x = a.x + (size_t)row * a.H;
    float ss = 0.f;
    for (int k = tid; k < a.H; k += 256) { const float v = bf2f(x[k]); ss += v * v; }
    ss = warp_sum(ss);
    if (lane == 0) red[0][warp] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < 8; w++) tot += red[0][w];
    const float inv = rsqrtf(tot / (float)a.H + a.eps);
    int step = 0;
    if (a.advance) step = a.st.step_counter[1];
    uint16_t* zo = a.z + (size_t)blockIdx.x * a.H;
    uint16_t* fo = a.feed ? a.feed + (size_t)blockIdx.x * a.H : nullptr;
    uint16_t* const ob = a.advance ? *a.st.out_cell : nullptr;
    float* const sb = a.advance ? *a.st.stop_cell : nullptr;
    uint16_t* oo = ob ? ob + ((size_t)step * gridDim.x + blockIdx.x) * a.H : nullptr;
    float l0 = 0.f, l1 = 0.f;
    for (int k = tid; k < a.H; k += 256) {
        const float z = rb(bf2f(a.nw[k]) * rb(bf2f(x[k]) * inv));
        const uint16_t zb = f2bf(z);
        zo[k] = zb;
        if (fo) fo[k] = zb;
        if (oo) oo[k] = zb;
        l0 += bf2f(a.ws[k]) * z;
        l1 += bf2f(a.ws[a.H + k]) * z;
    }
    l0 = warp_sum(l0);
    l1 = warp_sum(l1);
    __syncthreads();
    if (lane == 0) { red[1][warp] = l0; red[2][warp] = l1; }
    __syncthreads();
    if (tid == 0) {
        float a0 = 0.f, a1 = 0.f;
        for (int w = 0; w < 8; w++) { a0 += red[1][w]; a1 += red[2][w]; }
        a0 = rb(a0 + bf2f(a.bs[0]));
        a1 = rb(a1 + bf2f(a.bs[1]));
        const float m = fmaxf(a0, a1), e0 = expf(a0 - m), e1 = expf(a1 - m);
        const float p = e1 / (e0 + e1);
        a.stop[blockIdx.x] = p;
        if (a.advance) {
            if (sb) sb[(size_t)step * gridDim.x + blockIdx.x] = p;
            a.st.seq_len[a.st.row_seq[row]] += 1;
        }
    }
}

void launch_final(const FinalArgs& a, int rows, cudaStream_t s) { final_kernel<<<rows, 256, 0, s>>>(a); }

// Decode-step start: each row's position is its sequence's current length;
// snapshot the step counter for this step's output slot.
__global__ void step_begin_kernel(StepDev st, int rows) {
    const int r = threadIdx.x;
    if (r < rows) st.row_pos[r] = st.seq_len[st.row_seq[r]];
    if (r == 0) {
        st.step_counter[1] = st.step_counter[0];
        st.step_counter[0] += 1;
    }
}

void launch_step_begin(const StepDev& st, int rows, cudaStream_t s) { step_begin_kernel<<<1, 256, 0, s>>>(st, rows); }

}  // namespace ming
