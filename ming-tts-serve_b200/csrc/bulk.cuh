// bulk.cuh — the linear for decode batches (9..64 activation rows).
//
// A batched decode step moves every weight once and little else, but each
// projection is small (0.45-4.9 MB at 4 bits), so what decides its time is
// how many bytes are in flight while it starts. Here a CTA owns T tiles and a
// K range of them; its first thread bulk-copies all of those weights into
// shared memory (one cp.async.bulk per tile, the tile's K range being
// contiguous) BEFORE it waits on the previous kernel — the launch carries the
// programmatic-stream-serialization attribute, so the copies overlap the
// previous kernel's tail. After `griddepcontrol.wait` the CTA stages its K
// range of the activation rows (RMSNorm statistics over the whole row when
// the input is normed) as mma B fragments and lets the next kernel launch.
// The K ranges of one tile block form a thread-block cluster: partial sums
// meet over distributed shared memory, summed in rank order (deterministic),
// and the ranks split the epilogue.
//
// Numerics are those of linear_kernel / linear_frag_kernel (same operand
// rounding, same per-group scale and bias terms); only the f32 summation
// order of the K groups differs.
#pragma once

#include <cooperative_groups.h>

#include "linear.cuh"

namespace ming {

constexpr int BK_WARPS = 8;
constexpr int BK_THREADS = BK_WARPS * 32;
constexpr int BK_NT = 4;                     // 32 rows per CTA (zero rows are padding)
constexpr long long BK_TIMEOUT = 2000000000LL;  // cycles (~1 s) before the weight wait gives up
constexpr int BK_ERR_WEIGHTS = 7;            // device error code: weight copy never completed

struct BulkIn {
    const uint16_t* x;   // [rows][ld] bf16 activations
    const uint16_t* nw;  // RMSNorm gains [K] (normed input) or null (plain input)
    int ld;
    float eps;
    int* err;            // device error word
};

// Shared-memory layout of one CTA (bytes), for T tiles and up to gmax groups.
struct BulkSmem {
    int w, frag, ysum, red, part, aux, total;
    __host__ __device__ BulkSmem(int T, int gmax, int cb) {
        w = 128;
        frag = w + T * gmax * cb;
        ysum = frag + gmax * 4 * BK_NT * 32 * 8;
        red = ysum + gmax * 8 * BK_NT * 4;
        part = red + BK_WARPS * 16 * 8 * BK_NT * 4;
        aux = part + T * 16 * 8 * BK_NT * 4;
        total = aux + 2 * 8 * BK_NT * 4;
    }
};

MING_DEV uint32_t bk_saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MING_DEV bool bk_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t b = bk_saddr(bar);
    const long long t0 = clock64();
    while (true) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(b), "r"(parity)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > BK_TIMEOUT) return false;
    }
}

template <bool F16>
MING_DEV uint32_t bk_pack(float a, float b) {
    return F16 ? pack_f16x2(a, b) : pack_bf16x2(a, b);
}
template <bool F16>
MING_DEV float bk_sum2(uint32_t u) {
    if (F16) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&u));
        return v.x + v.y;
    }
    const float2 v = unpack_bf16x2(u);
    return v.x + v.y;
}

// Grid: x = tile block * ks + rank (cluster (ks, 1, 1)), y = 32-row block.
template <int FMT, int T, bool RMS, class Epi>
__global__ void __launch_bounds__(BK_THREADS) linear_bulk_kernel(PackedW W, BulkIn in, Epi epi, int rows, int ks, int gmax) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int CB = chunk_b(FMT), NT = BK_NT;
    constexpr bool F16 = FMT != 16;
    const BulkSmem L(T, gmax, CB);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    uint8_t* wbuf = smem + L.w;
    uint2* sB = reinterpret_cast<uint2*>(smem + L.frag);
    float* sYs = reinterpret_cast<float*>(smem + L.ysum);
    float* sRed = reinterpret_cast<float*>(smem + L.red);
    float* sPart = reinterpret_cast<float*>(smem + L.part);
    float* sAux = reinterpret_cast<float*>(smem + L.aux);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = blockIdx.x % ks, tile0 = (blockIdx.x / ks) * T;
    const int ng = W.K / 64;
    const int g0 = rank * ng / ks, gc = (rank + 1) * ng / ks - g0;
    const int r0 = blockIdx.y * 8 * NT, nrows = min(8 * NT, rows - r0);
    const int nt = min(T, W.ntiles - tile0);

    // 1. this CTA's weights, before waiting on the previous kernel
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bk_saddr(bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bk_saddr(bar)),
                     "r"((uint32_t)(nt * gc * CB))
                     : "memory");
        for (int t = 0; t < nt; t++)
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                             bk_saddr(wbuf + (size_t)t * gmax * CB)),
                         "l"(W.tiles + ((size_t)(tile0 + t) * ng + g0) * CB), "r"((uint32_t)(gc * CB)), "r"(bk_saddr(bar))
                         : "memory");
    }
    // 2. the activations are the previous kernel's output
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    // 3. RMSNorm statistics over the whole row (ProRms::init's values): warp w
    //    takes rows w, w + 8, w + 16, w + 24, 16-byte pieces, 16 loads in flight
    if (RMS) {
        const int npr = W.K / 8;
        float s[4] = {0.f, 0.f, 0.f, 0.f}, amax[4] = {0.f, 0.f, 0.f, 0.f};
        for (int j0 = 0; j0 < npr; j0 += 128) {
            uint4 v[4][4], w[4];
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const int p = j0 + lane + 32 * jj;
                w[jj] = p < npr ? *reinterpret_cast<const uint4*>(in.nw + p * 8) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int r = warp + 8 * i;
                    v[i][jj] = p < npr && r < nrows ? *reinterpret_cast<const uint4*>(in.x + (size_t)(r0 + r) * in.ld + p * 8)
                                                    : make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                const uint32_t ww[4] = {w[jj].x, w[jj].y, w[jj].z, w[jj].w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const uint32_t xx[4] = {v[i][jj].x, v[i][jj].y, v[i][jj].z, v[i][jj].w};
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        const float2 a = unpack_bf16x2(xx[q]), b = unpack_bf16x2(ww[q]);
                        s[i] += a.x * a.x + a.y * a.y;
                        amax[i] = fmaxf(amax[i], fmaxf(fabsf(a.x * b.x), fabsf(a.y * b.y)));
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float ss = warp_sum(s[i]), am = warp_max(amax[i]);
            const int r = warp + 8 * i;
            if (lane == 0 && r < nrows) {
                int e = 0;
                if (F16 && am > 4096.f) frexpf(am / 4096.f, &e);  // 2^e >= amax / 4096
                sAux[2 * r] = ldexpf(1.f, -e);
                sAux[2 * r + 1] = rsqrtf(ss / (float)W.K + in.eps) * ldexpf(1.f, e);
            }
        }
        __syncthreads();
    }
    // 4. B fragments of K range [64 g0, 64 (g0 + gc)) for 32 rows, 8 pieces of
    //    8 values per thread in flight. Piece (row, k..k+7) fills the .x (k % 16
    //    == 0) or .y half of entries lane 4 (row % 8) + t, t = 0..3. A warp
    //    takes one 64-group of 4 rows (8 pieces per row in 8 consecutive
    //    lanes: their shuffle sum is the group's operand sum; 128-byte row
    //    segments from global memory; 4-way bank overlap on the stores).
    {
        const int tot = 8 * NT * gc * 8, kc0 = g0 * 64;  // 256 gc: e < tot is uniform over the CTA
        for (int e0 = tid; e0 < tot; e0 += 8 * BK_THREADS) {
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int e = e0 + u * BK_THREADS, b = e >> 5;
                const int row = (b & 7) * 4 + ((e >> 3) & 3), k = ((b >> 3) * 8 + (e & 7)) * 8;
                v[u] = e < tot && row < nrows ? *reinterpret_cast<const uint4*>(in.x + (size_t)(r0 + row) * in.ld + kc0 + k)
                                              : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int e = e0 + u * BK_THREADS, b = e >> 5;
                if (e >= tot) break;
                const int row = (b & 7) * 4 + ((e >> 3) & 3), k = ((b >> 3) * 8 + (e & 7)) * 8;
                float y[8];
                const uint32_t vv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 f = unpack_bf16x2(vv[i]);
                    y[2 * i] = f.x;
                    y[2 * i + 1] = f.y;
                }
                if (RMS && row < nrows) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(in.nw + kc0 + k);
                    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
                    const float sc = sAux[2 * row];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float2 f = unpack_bf16x2(ww[i]);
                        y[2 * i] = y[2 * i] * f.x * sc;
                        y[2 * i + 1] = y[2 * i + 1] * f.y * sc;
                    }
                }
                uint32_t* dst = reinterpret_cast<uint32_t*>(sB + ((size_t)(k >> 4) * NT + (row >> 3)) * 32 + 4 * (row & 7)) +
                                ((k >> 3) & 1);
                float s = 0.f;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const uint32_t pk = bk_pack<F16>(y[2 * t], y[2 * t + 1]);
                    dst[2 * t] = pk;
                    s += bk_sum2<F16>(pk);
                }
                if (F16) {
                    s += __shfl_xor_sync(0xffffffffu, s, 1);
                    s += __shfl_xor_sync(0xffffffffu, s, 2);
                    s += __shfl_xor_sync(0xffffffffu, s, 4);
                    if ((lane & 7) == 0) sYs[(k >> 6) * 8 * NT + row] = s;
                }
            }
        }
    }
    __syncthreads();
    // the next kernel may launch and start its own weight copies
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    // 5. weights landed?
    if (!bk_wait(bar, 0) && tid == 0) atomicCAS(in.err, 0, BK_ERR_WEIGHTS);
    // 6. warp w: tile w % T, groups w / T, + 8 / T, ...
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    {
        const int t = warp % T;
        if (t < nt) {
#pragma unroll 2
            for (int gi = warp / T; gi < gc; gi += BK_WARPS / T)
                group_mma<FMT, NT, true>(wbuf + ((size_t)t * gmax + gi) * CB, sB + (size_t)gi * 4 * NT * 32,
                                         sYs + gi * 8 * NT, acc, lane);
        }
    }
    {
        const int g = lane >> 2, c = 2 * (lane & 3);
        float* r = sRed + warp * 16 * 8 * NT;
#pragma unroll
        for (int j = 0; j < NT; j++) {
            r[g * 8 * NT + j * 8 + c] = acc[j][0];
            r[g * 8 * NT + j * 8 + c + 1] = acc[j][1];
            r[(g + 8) * 8 * NT + j * 8 + c] = acc[j][2];
            r[(g + 8) * 8 * NT + j * 8 + c + 1] = acc[j][3];
        }
    }
    __syncthreads();
    // per tile: the sum of its warps, in warp order
    for (int e = tid; e < T * 16 * 8 * NT; e += BK_THREADS) {
        const int t = e / (16 * 8 * NT), rc = e - t * 16 * 8 * NT;
        float s = 0.f;
        for (int w = t; w < BK_WARPS; w += T) s += sRed[w * 16 * 8 * NT + rc];
        sPart[e] = s;
    }
    // 7. the ks ranks' partials, summed in rank order; rank r takes every
    //    ks-th (tile, row pair, activation row)
    cg::cluster_group cl = cg::this_cluster();
    if (ks > 1) cl.sync();
    else __syncthreads();
    for (int e = rank * BK_THREADS + tid; e < T * 8 * 8 * NT; e += ks * BK_THREADS) {
        const int t = e / (64 * NT), rem = e - t * 64 * NT, r8 = rem / (8 * NT), col = rem - r8 * 8 * NT;
        if (t >= nt || col >= nrows) continue;
        float lo = 0.f, hi = 0.f;
        for (int q = 0; q < ks; q++) {
            const float* pq = ks > 1 ? cl.map_shared_rank(sPart, q) : sPart;
            lo += pq[(t * 16 + r8) * 8 * NT + col];
            hi += pq[(t * 16 + r8 + 8) * 8 * NT + col];
        }
        const float ps = RMS ? sAux[2 * col + 1] : 1.f;
        epi(tile0 + t, r8, r0 + col, lo * ps, hi * ps);
    }
    // peers may still be reading this CTA's partials
    if (ks > 1) cl.sync();
}

// ---------------- host side ----------------

struct BulkPlan {
    int T = 1, ks = 1, gmax = 0, smem = 0;
};

constexpr int BK_SMEM_MAX = 200 * 1024;

// Picks T (4 or 1 tiles per CTA) and the K split (1..8 ranks): the fewest
// waves of resident CTAs, then at least one CTA per SM, then the fewest
// ranks, then the larger T. Residency from shared memory and the kernels'
// register counts (regs[0]: T = 4, regs[1]: T = 1).
inline BulkPlan bulk_plan(int ntiles, int K, int rows, int fmt, int sms, const int (&regs)[2]) {
    const int ng = K / 64, cb = fmt == 4 ? 576 : (fmt == 8 ? 1088 : 2048);
    const long rb = (rows + 8 * BK_NT - 1) / (8 * BK_NT);
    BulkPlan best;
    long bw = 0, bs = 0, bk = 0;
    bool have = false;
    for (int i = 0; i < 2; i++) {
        const int T = i == 0 ? 4 : 1;
        const int rg = (std::max(regs[i], 32) + 7) / 8 * 8;
        for (int ks = 1; ks <= 8 && ks <= ng; ks++) {
            BulkPlan p;
            p.T = T;
            p.ks = ks;
            p.gmax = (ng + ks - 1) / ks;
            p.smem = BulkSmem(T, p.gmax, cb).total;
            if (p.smem > BK_SMEM_MAX) continue;
            const long occ = std::max(1L, std::min({8L, 65536L / (rg * BK_THREADS), (long)(228 * 1024) / (p.smem + 1024)}));
            const long ctas = (long)((ntiles + T - 1) / T) * ks * rb;
            const long waves = (ctas + sms * occ - 1) / (sms * occ);
            const long shortfall = ctas < sms ? 1 : 0;
            if (!have || waves < bw || (waves == bw && (shortfall < bs || (shortfall == bs && ks < bk)))) {
                best = p;
                bw = waves;
                bs = shortfall;
                bk = ks;
                have = true;
            }
        }
    }
    return best;
}

template <int FMT, int T, bool RMS, class Epi>
int bulk_regs() {
    static int r = 0;
    if (!r) {
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, linear_bulk_kernel<FMT, T, RMS, Epi>) == cudaSuccess) r = fa.numRegs;
        else r = 128;
    }
    return r;
}

template <int FMT, int T, bool RMS, class Epi>
cudaError_t launch_bulk_t(const PackedW& W, const BulkIn& in, const Epi& e, int rows, const BulkPlan& p, cudaStream_t s) {
    static unsigned attr_devices = 0;  // bit d: attribute set on device d
    auto kern = linear_bulk_kernel<FMT, T, RMS, Epi>;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_devices & (1u << (dev & 31)))) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BK_SMEM_MAX);
        attr_devices |= 1u << (dev & 31);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((W.ntiles + T - 1) / T) * p.ks), (unsigned)((rows + 8 * BK_NT - 1) / (8 * BK_NT)));
    cfg.blockDim = dim3(BK_THREADS);
    cfg.dynamicSmemBytes = (size_t)p.smem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = (unsigned)p.ks;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = p.ks > 1 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, W, in, e, rows, p.ks, p.gmax);
}

template <int FMT, bool RMS, class Epi>
cudaError_t launch_bulk(const PackedW& W, const BulkIn& in, const Epi& e, int rows, int sms, cudaStream_t s) {
    const int regs[2] = {bulk_regs<FMT, 4, RMS, Epi>(), bulk_regs<FMT, 1, RMS, Epi>()};
    const BulkPlan p = bulk_plan(W.ntiles, W.K, rows, FMT, sms, regs);
    if (p.T == 4) return launch_bulk_t<FMT, 4, RMS>(W, in, e, rows, p, s);
    return launch_bulk_t<FMT, 1, RMS>(W, in, e, rows, p, s);
}

}  // namespace ming
