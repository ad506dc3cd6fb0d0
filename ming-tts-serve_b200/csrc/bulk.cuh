// bulk.cuh — the linear for decode batches (9..64 activation rows).
//
// A batched decode step moves every weight once and little else, but each
// projection is small (0.45-4.9 MB at 4 bits): its time is a chain of
// latencies, so this kernel keeps the chain short.
//
//  * One CTA per SM (16 warps). A CTA owns a balanced range of tiles and a K
//    range of them; the K ranges of one tile range form a thread-block
//    cluster whose partial sums meet over distributed shared memory, summed
//    in rank order (deterministic), the ranks splitting the epilogue.
//  * The first thread bulk-copies the CTA's weights (one cp.async.bulk per
//    tile: a tile's K range is contiguous) BEFORE `griddepcontrol.wait`: the
//    launch is a programmatic dependent of the previous kernel, so the copies
//    overlap its tail. After the wait it bulk-copies the K range of each
//    activation row, raw bf16, into a row-major shared array whose row
//    stride is 4 words mod 32 — the mma B fragments are read from it without
//    bank conflicts and without any staging pass.
//  * The tensor cores run bf16 x bf16 -> f32: 4- and 8-bit codes become exact
//    bf16 integers in registers, the per-group scale and bias are applied in
//    f32 (s * sum(q y) + b * sum(y)), sum(y) of each 64-group and row
//    computed once per CTA.
//  * Input prologues (PRO): BK_PLAIN rows as they are; BK_LNMOD LayerNorm
//    (no affine, eps 1e-6) + adaLN modulation, rb(LN(x) (1 + scale) + shift)
//    with ProLnMod's statistics order, applied to the staged rows in place
//    (K unsplit); BK_RMS as follows.
//  * RMSNorm inputs: each rank sums x^2 over its K range; the epilogue adds
//    the ranks' sums (rank order) and applies rsqrt(mean + eps) to the f32
//    dot products, as the reference's fused kernels fold the norm
//    (src/ming_fused.zig:100-142). With non-unit gains the f32 product
//    x * g enters the mma as two bf16 parts, hi + lo (~16 significant bits).
#pragma once

#include <cuda_bf16.h>

#include <algorithm>
#include <cooperative_groups.h>

#include "linear.cuh"
#include "tcgen05.cuh"

namespace ming {

constexpr int BK_WARPS = 16;
constexpr int BK_THREADS = BK_WARPS * 32;
constexpr int BK_ROWS = 32;                     // activation rows per CTA (4 mma n-tiles)
constexpr int BK_TMAX = 8;                      // tiles per CTA at most
constexpr int BK_SMEM_MAX = 200 * 1024;
constexpr int BK_SMEM_TC_MAX = 226 * 1024;
constexpr long long BK_TIMEOUT = 2000000000LL;  // cycles (~1 s) before a copy wait gives up
constexpr int BK_ERR_WEIGHTS = 7;               // device error code: a bulk copy never completed

constexpr int BK_PLAIN = 0, BK_RMS = 1, BK_LNMOD = 2;

struct BulkIn {
    const uint16_t* x;   // [rows][ld] bf16 activations
    const uint16_t* nw;  // RMSNorm gains [K] when not all 1, else null
    int ld;
    float eps;
    int* err;            // device error word
    long long* trace = nullptr;  // launch trace: [CTA][8] globaltimer stamps (entry, wait done, rows in, sums done,
                                 // weights in, mma done, cluster met, exit) or null
    // BK_LNMOD: modulation rows [cond][mod_ld]; condition of row r = r / rpc
    const uint16_t* shift = nullptr;
    const uint16_t* scale = nullptr;
    int mod_ld = 0, rpc = 1;
};

// Shared-memory layout of one CTA (bytes): barriers, tensor-memory slot and
// per-row x^2 sums; per-(group, row) operand sums and x^2 sums [gmax][32]
// each; with TC the two 1024-aligned stages of the tcgen05 operands (weight
// block 128 x 64 bf16, row block 32 x 64 bf16 (+ low parts)); packed weights
// [tmax][gmax][chunk]; staged rows [32 (+ 32 low parts)][gmax * 64 + 8] bf16
// (reused for the warps' partial sums after the mma.sync loop); per-tile
// sums [tmax * 16][32]. With TC the kernel aligns its base up to 1024 bytes
// (the slack is in `total`).
struct BulkSmem {
    int ss, ys, xx, a, b, w, x, xstride, part, total;
    __host__ __device__ BulkSmem(int tmax, int gmax, int cb, bool lo, bool tc = false) {
        ss = 128;
        ys = 256;
        xx = ys + gmax * BK_ROWS * 4;
        a = b = 0;
        w = xx + gmax * BK_ROWS * 4;
        if (tc) {
            a = (w + 1023) / 1024 * 1024;
            const int nst = lo ? 2 : 4;  // operand stages (4 hide the MMA round trip; 2 leave room for low parts)
            b = a + nst * TC_A_BLOCK;
            w = b + nst * (lo ? 2 : 1) * BK_ROWS * 128;
        }
        x = w + tmax * gmax * cb;
        xstride = gmax * 128 + 16;
        const int xb = (lo ? 2 : 1) * BK_ROWS * xstride, red = tc ? 0 : BK_WARPS * 16 * BK_ROWS * 4;
        part = x + (xb > red ? xb : red);
        total = part + tmax * 16 * BK_ROWS * 4 + (tc ? 1024 : 0);
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

MING_DEV void bk_bulk(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     bk_saddr(dst)),
                 "l"(src), "r"(bytes), "r"(bk_saddr(bar))
                 : "memory");
}

MING_DEV uint32_t bsub2_u(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// 4-bit codes of one m16k16 step (the word layout dq4 reads) as exact bf16
// integers: (nibble | 0x4300) is 128 + nibble.
MING_DEV void dq4_bf16(uint32_t u, uint32_t (&a)[4]) {
    const uint32_t MAGIC = 0x43004300u;  // bf16x2(128, 128)
    a[0] = bsub2_u(lop3<(0xF0 & 0xCC) | 0xAA>(u, 0x000F000Fu, MAGIC), MAGIC);
    a[1] = bsub2_u(lop3<(0xF0 & 0xCC) | 0xAA>(u >> 4, 0x000F000Fu, MAGIC), MAGIC);
    a[2] = bsub2_u(lop3<(0xF0 & 0xCC) | 0xAA>(u >> 8, 0x000F000Fu, MAGIC), MAGIC);
    a[3] = bsub2_u(lop3<(0xF0 & 0xCC) | 0xAA>(u >> 12, 0x000F000Fu, MAGIC), MAGIC);
}

// 8-bit codes (the word layout dq8 reads) as exact bf16 integers, through
// f32: (byte | 0x4B000000) is 2^23 + byte.
MING_DEV uint32_t b8pair(uint32_t w, uint32_t s0, uint32_t s1) {
    const float f0 = __uint_as_float(__byte_perm(w, 0x4B000000u, s0)) - 8388608.f;
    const float f1 = __uint_as_float(__byte_perm(w, 0x4B000000u, s1)) - 8388608.f;
    return pack_bf16x2(f0, f1);
}
MING_DEV void dq8_bf16(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    a[0] = b8pair(w0, 0x7440u, 0x7441u);
    a[1] = b8pair(w0, 0x7442u, 0x7443u);
    a[2] = b8pair(w1, 0x7440u, 0x7441u);
    a[3] = b8pair(w1, 0x7442u, 0x7443u);
}

// One 64-group of one tile over the 32 staged rows: acc[j] += W_group . y
// for n-tile j (rows 8j..8j+7). xs: the staged rows as 32-bit words, at the
// group's first column; xw: words per staged row; ys: the group's operand
// sums per row.
template <int FMT>
MING_DEV void bk_group(const uint8_t* chunk, const uint32_t* xs, int xw, bool lo, int ntl, const float* ys, float (&acc)[4][4],
                       int lane) {
    const int g = lane >> 2, t = lane & 3;
    if constexpr (FMT == 16) {
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            const uint4 w = *reinterpret_cast<const uint4*>(chunk + ((size_t)ks * 32 + lane) * 16);
            const uint32_t a[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (j >= ntl) break;
                const uint32_t* b = xs + (j * 8 + g) * xw + ks * 8 + t;
                mma_bf16(acc[j], a, b[0], b[4]);
                if (lo) mma_bf16(acc[j], a, b[BK_ROWS * xw], b[BK_ROWS * xw + 4]);
            }
        }
    } else {
        uint32_t words[8];
        if constexpr (FMT == 4) {
            const uint4 w = *reinterpret_cast<const uint4*>(chunk + (size_t)lane * 16);
            words[0] = w.x; words[1] = w.y; words[2] = w.z; words[3] = w.w;
        } else {
            const uint4 w0 = *reinterpret_cast<const uint4*>(chunk + (size_t)lane * 16);
            const uint4 w1 = *reinterpret_cast<const uint4*>(chunk + (size_t)(32 + lane) * 16);
            words[0] = w0.x; words[1] = w0.y; words[2] = w0.z; words[3] = w0.w;
            words[4] = w1.x; words[5] = w1.y; words[6] = w1.z; words[7] = w1.w;
        }
        const uint2 sc = *reinterpret_cast<const uint2*>(chunk + (FMT == 4 ? 512 : 1024) + g * 8);
        const float s_lo = __uint_as_float(sc.x << 16), b_lo = __uint_as_float(sc.x & 0xffff0000u);
        const float s_hi = __uint_as_float(sc.y << 16), b_hi = __uint_as_float(sc.y & 0xffff0000u);
        float tq[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int i = 0; i < 4; i++) tq[j][i] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            uint32_t a[4];
            if constexpr (FMT == 4) dq4_bf16(words[ks], a);
            else dq8_bf16(words[(ks >> 1) * 4 + (ks & 1) * 2], words[(ks >> 1) * 4 + (ks & 1) * 2 + 1], a);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (j >= ntl) break;
                const uint32_t* b = xs + (j * 8 + g) * xw + ks * 8 + t;
                mma_bf16(tq[j], a, b[0], b[4]);
                if (lo) mma_bf16(tq[j], a, b[BK_ROWS * xw], b[BK_ROWS * xw + 4]);
            }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 y = *reinterpret_cast<const float2*>(ys + j * 8 + 2 * t);
            acc[j][0] += s_lo * tq[j][0] + b_lo * y.x;
            acc[j][1] += s_lo * tq[j][1] + b_lo * y.y;
            acc[j][2] += s_hi * tq[j][2] + b_hi * y.x;
            acc[j][3] += s_hi * tq[j][3] + b_hi * y.y;
        }
    }
}

// Grid: x = tile range * ks + rank (cluster (ks, 1, 1)), y = 32-row block.
// TC: the tile range is one block of 8 tiles (128 features) and the products
// run on tcgen05 (see the TC section below); otherwise on mma.sync.
template <int FMT, int PRO, bool TC, class Epi>
__global__ void __launch_bounds__(BK_THREADS, 1)
    linear_bulk_kernel(PackedW W, BulkIn in, Epi epi, int rows, int ks, int nb, int tmax, int gmax) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // TC: 1024-byte aligned base (the swizzle atoms of the tcgen05 operands)
    uint8_t* smem = TC ? smem_raw + ((1024u - (bk_saddr(smem_raw) & 1023u)) & 1023u) : smem_raw;
    constexpr int CB = chunk_b(FMT);
    constexpr bool RMS = PRO == BK_RMS;
    const bool lo = RMS && in.nw;  // non-unit gains: the normed operand is hi + lo (two bf16 parts)
    const BulkSmem L(tmax, gmax, CB, lo, TC);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);  // [0] weights, [1] rows; TC: [2..5] stages read, [6] mma done
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + 64);  // TC: tensor-memory base
    float* sSS = reinterpret_cast<float*>(smem + L.ss);  // [32] this rank's x^2 sums (RMS)
    float* sYs = reinterpret_cast<float*>(smem + L.ys);  // [gmax][32] operand sums (quantized formats)
    uint8_t* wbuf = smem + L.w;
    uint16_t* sX = reinterpret_cast<uint16_t*>(smem + L.x);
    float* sRed = reinterpret_cast<float*>(smem + L.x);  // after the mma loop
    float* sPart = reinterpret_cast<float*>(smem + L.part);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = blockIdx.x % ks, blk = blockIdx.x / ks;
    const int tile0 = blk * W.ntiles / nb, nt = (blk + 1) * W.ntiles / nb - tile0;
    const int ng = W.K / 64;
    const int g0 = rank * ng / ks, gc = (rank + 1) * ng / ks - g0;
    const int r0 = blockIdx.y * BK_ROWS, nrows = min(BK_ROWS, rows - r0);
    const int xs_b = L.xstride;

    long long* tr = in.trace && tid == 0 ? in.trace + ((size_t)blockIdx.y * gridDim.x + blockIdx.x) * 8 : nullptr;
    if (tr) tr[0] = gtimer();
    // 1. this CTA's weights, before the wait on the previous kernel
    // TC: tensor memory for one 32-column accumulator per K group (gc <= 16)
    const uint32_t tcols = gc <= 1 ? 32u : (gc <= 2 ? 64u : (gc <= 4 ? 128u : (gc <= 8 ? 256u : 512u)));
    if (TC && warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(bk_saddr(tslot)), "r"(tcols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bk_saddr(&bar[0])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bk_saddr(&bar[1])) : "memory");
        if (TC)
            for (int i = 2; i < 7; i++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(bk_saddr(&bar[i])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bk_saddr(&bar[0])),
                     "r"((uint32_t)(nt * gc * CB))
                     : "memory");
        for (int t = 0; t < nt; t++)
            bk_bulk(wbuf + (size_t)t * gmax * CB, W.tiles + ((size_t)(tile0 + t) * ng + g0) * CB, (uint32_t)(gc * CB),
                    &bar[0]);
    }
    if (TC) asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();  // the barriers are initialised before anyone waits on them
    if (TC) asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    // 2. the activation rows are the previous kernel's output
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (tr) tr[1] = gtimer();
    if (warp == 0) {  // one row per lane: every copy in flight at once
        if (lane == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bk_saddr(&bar[1])),
                         "r"((uint32_t)(nrows * gc * 128))
                         : "memory");
        __syncwarp();
        if (lane < nrows)
            bk_bulk(reinterpret_cast<uint8_t*>(sX) + (size_t)lane * xs_b, in.x + (size_t)(r0 + lane) * in.ld + g0 * 64,
                    (uint32_t)(gc * 128), &bar[1]);
    }
    // rows past the batch in the n-tiles used (and their low parts) are zero
    const int ntl = TC ? 4 : (nrows + 7) / 8;  // TC: the mma reads all 32 rows
    for (int e = nrows * gc * 8 + tid; e < ntl * 8 * gc * 8; e += BK_THREADS) {
        const int r = e / (gc * 8), c = e - r * gc * 8;
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sX) + (size_t)r * xs_b + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        if (lo)
            *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sX) + (size_t)(BK_ROWS + r) * xs_b + c * 16) =
                make_uint4(0u, 0u, 0u, 0u);
    }
    bool ok = bk_wait(&bar[1], 0);
    if (tr) tr[2] = gtimer();
    if constexpr (PRO == BK_LNMOD) {
        // LayerNorm statistics of each row (ProLnMod::init's order: lanes
        // stride the row, then the warp sum), then the modulated operand in place
        float* sMu = sSS;                                     // [32]
        float* sInv = reinterpret_cast<float*>(smem + L.xx);  // [32]
        for (int r = warp; r < nrows; r += BK_WARPS) {
            const uint16_t* xr = reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(sX) + (size_t)r * xs_b);
            float sm = 0.f;
            for (int k = lane; k < W.K; k += 32) sm += bf2f(xr[k]);
            const float mu = warp_sum(sm) / (float)W.K;
            float v = 0.f;
            for (int k = lane; k < W.K; k += 32) {
                const float d = bf2f(xr[k]) - mu;
                v += d * d;
            }
            v = warp_sum(v) / (float)W.K;
            if (lane == 0) {
                sMu[r] = mu;
                sInv[r] = rsqrtf(v + 1e-6f);
            }
        }
        __syncthreads();
        for (int e = tid; e < nrows * gc * 8; e += BK_THREADS) {
            const int r = e / (gc * 8), c = e - r * gc * 8, k = c * 8;
            uint4* xp = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sX) + (size_t)r * xs_b) + c;
            const uint4 v = *xp;
            const size_t mo = (size_t)((r0 + r) / in.rpc) * in.mod_ld + k;
            const uint4 sc4 = *reinterpret_cast<const uint4*>(in.scale + mo), sh4 = *reinterpret_cast<const uint4*>(in.shift + mo);
            const uint32_t vv[4] = {v.x, v.y, v.z, v.w}, cc[4] = {sc4.x, sc4.y, sc4.z, sc4.w}, hh[4] = {sh4.x, sh4.y, sh4.z, sh4.w};
            const float mu = sMu[r], iv = sInv[r];
            uint32_t out[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f = unpack_bf16x2(vv[i]), sc2 = unpack_bf16x2(cc[i]), sh2 = unpack_bf16x2(hh[i]);
                const float n0 = (f.x - mu) * iv, n1 = (f.y - mu) * iv;
                out[i] = pack_bf16x2(rb(n0 * (1.0f + sc2.x) + sh2.x), rb(n1 * (1.0f + sc2.y) + sh2.y));
            }
            *xp = make_uint4(out[0], out[1], out[2], out[3]);
        }
        __syncthreads();
    }
    // 3. one pass over the staged rows, a thread per (64-group, row): the
    //    operand sum of the group (the bias term of the quantized formats)
    //    and, for RMSNorm inputs, the group's x^2 sum; with non-unit gains
    //    the f32 product x * g is kept as hi = bf16(x g) in place and
    //    lo = bf16(x g - hi) in row 32 + r (both go through the mma). Row
    //    x^2 sums add the groups in order.
    if (FMT != 16 || RMS) {
        float* sXX = reinterpret_cast<float*>(smem + L.xx);  // [gmax][32] per-group x^2
        for (int e = tid; e < gc * BK_ROWS; e += BK_THREADS) {
            const int gi = e / BK_ROWS, r = e - gi * BK_ROWS;
            uint8_t* xr = reinterpret_cast<uint8_t*>(sX) + (size_t)r * xs_b + gi * 128;
            uint4 v[8];
#pragma unroll
            for (int c = 0; c < 8; c++) v[c] = reinterpret_cast<const uint4*>(xr)[c];
            float sy[2] = {0.f, 0.f}, sx[2] = {0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 8; c++) {
                uint32_t vv[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
                if (lo && r < nrows) {
                    const uint4 wv = *reinterpret_cast<const uint4*>(in.nw + (g0 + gi) * 64 + c * 8);
                    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
                    uint32_t ll[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float2 f = unpack_bf16x2(vv[i]), w = unpack_bf16x2(ww[i]);
                        sx[i & 1] += f.x * f.x + f.y * f.y;
                        const float px = f.x * w.x, py = f.y * w.y;
                        const uint32_t h = pack_bf16x2(px, py);
                        const float2 hf = unpack_bf16x2(h);
                        ll[i] = pack_bf16x2(px - hf.x, py - hf.y);
                        const float2 lf = unpack_bf16x2(ll[i]);
                        sy[i & 1] += (hf.x + hf.y) + (lf.x + lf.y);
                        vv[i] = h;
                    }
                    reinterpret_cast<uint4*>(xr)[c] = make_uint4(vv[0], vv[1], vv[2], vv[3]);
                    reinterpret_cast<uint4*>(xr + (size_t)BK_ROWS * xs_b)[c] = make_uint4(ll[0], ll[1], ll[2], ll[3]);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float2 f = unpack_bf16x2(vv[i]);
                        sy[i & 1] += f.x + f.y;
                        sx[i & 1] += f.x * f.x + f.y * f.y;
                    }
                }
            }
            sYs[gi * BK_ROWS + r] = sy[0] + sy[1];
            if (RMS) sXX[gi * BK_ROWS + r] = sx[0] + sx[1];
        }
        __syncthreads();
        if (RMS && tid < nrows) {
            float ss = 0.f;
            for (int gi = 0; gi < gc; gi++) ss += sXX[gi * BK_ROWS + tid];
            sSS[tid] = ss;
        }
    }
    __syncthreads();
    if (tr) tr[3] = gtimer();
    // the next kernel may launch and start its own weight copies
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    ok = bk_wait(&bar[0], 0) && ok;
    if (tr) tr[4] = gtimer();
    if (!ok && tid == 0) atomicCAS(in.err, 0, BK_ERR_WEIGHTS);
    if constexpr (TC) {
        // 4. tcgen05: per K group, every thread writes its share of the 128 x 64
        //    weight block (codes -> exact bf16, 128-byte-swizzled K-major, the
        //    layout tc_swizzle_kernel gives bf16 weights) and of the 32 x 64 row
        //    block into one of two stages; after a proxy fence and a barrier
        //    one thread issues 4 tcgen05.mma (M 128, N 32, K 16) into the
        //    group's own 32 tensor-memory columns and commits to the stage's
        //    barrier, so the group scale and bias stay in f32 (below).
        uint64_t* mbar = bar + 2;
        uint64_t* dbar = bar + 6;
        const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);
        const int bstage = (lo ? 2 : 1) * BK_ROWS * 128, nst = lo ? 2 : 4, lst = lo ? 1 : 2;
        bool tok = ok;
        for (int gi = 0; gi < gc; gi++) {
            const int s = gi & (nst - 1);  // the stage of group gi - nst must have been read
            if (gi >= nst && !bk_wait(&mbar[s], ((gi >> lst) - 1) & 1)) tok = false;
            uint8_t* A = smem + L.a + s * TC_A_BLOCK;
            uint8_t* Bs = smem + L.b + s * bstage;
            for (int e = tid; e < 8 * 32 * 4; e += BK_THREADS) {
                const int tt = e >> 7, ln = (e >> 2) & 31, kq = e & 3;
                const uint8_t* ch = wbuf + ((size_t)tt * gmax + gi) * CB;
                uint32_t av[4];
                if constexpr (FMT == 4) {
                    dq4_bf16(reinterpret_cast<const uint32_t*>(ch + ln * 16)[kq], av);
                } else if constexpr (FMT == 8) {
                    const uint32_t* wp = reinterpret_cast<const uint32_t*>(ch + ((kq >> 1) * 32 + ln) * 16) + (kq & 1) * 2;
                    dq8_bf16(wp[0], wp[1], av);
                } else {
                    const uint4 w = reinterpret_cast<const uint4*>(ch)[kq * 32 + ln];
                    av[0] = w.x; av[1] = w.y; av[2] = w.z; av[3] = w.w;
                }
                // lane (g, t): (row g, k 16 kq + 2t..+1), (row g + 8, same), (row g, +8), (row g + 8, +8)
                const int m0 = tt * 16 + (ln >> 2), t4 = (ln & 3) * 4;
                *reinterpret_cast<uint32_t*>(A + tc_sw128(m0, 2 * kq) + t4) = av[0];
                *reinterpret_cast<uint32_t*>(A + tc_sw128(m0 + 8, 2 * kq) + t4) = av[1];
                *reinterpret_cast<uint32_t*>(A + tc_sw128(m0, 2 * kq + 1) + t4) = av[2];
                *reinterpret_cast<uint32_t*>(A + tc_sw128(m0 + 8, 2 * kq + 1) + t4) = av[3];
            }
            for (int e = tid; e < (lo ? 2 : 1) * BK_ROWS * 8; e += BK_THREADS) {
                const int part = e >> 8, n = (e >> 3) & 31, c = e & 7;
                const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(sX) +
                                                                (size_t)(part * BK_ROWS + n) * xs_b + gi * 128 + c * 16);
                *reinterpret_cast<uint4*>(Bs + part * BK_ROWS * 128 + tc_sw128(n, c)) = v;
            }
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // thread writes -> tensor-core reads
            __syncthreads();
            if (tid == 0) {
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
                const uint32_t a0 = bk_saddr(A), b0 = bk_saddr(Bs);
#pragma unroll
                for (int kq = 0; kq < 4 * 2; kq++) {
                    if (kq >= 4 && !lo) break;
                    const uint64_t da = tc_desc(a0 + 32 * (kq & 3)), db = tc_desc(b0 + (kq >> 2) * BK_ROWS * 128 + 32 * (kq & 3));
                    const uint32_t accf = kq > 0 ? 1u : 0u;
                    asm volatile(
                        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem + (uint32_t)(gi * 32)),
                        "l"(da), "l"(db), "r"(tc_idesc<BK_ROWS>()), "r"(accf)
                        : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                                 bk_saddr(&mbar[s]))
                             : "memory");
            }
        }
        if (tid == 0)
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bk_saddr(dbar))
                         : "memory");
        tok = bk_wait(dbar, 0) && tok;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        if (!tok && tid == 0) atomicCAS(in.err, 0, BK_ERR_WEIGHTS);
        if (tr) tr[5] = gtimer();
        // the groups' accumulators, scaled in f32: warp w reads tensor-memory
        // lanes 32 (w % 4) .. (feature m = its lane) and rows 8 (w / 4) .. + 8
        {
            const int q = warp & 3, cb = warp >> 2, m = q * 32 + lane, tt = m >> 4, rr = m & 15;
            float av[8];
#pragma unroll
            for (int j = 0; j < 8; j++) av[j] = 0.f;
            // four groups' loads in flight per wait
            for (int g4 = 0; g4 < gc; g4 += 4) {
                uint32_t v[4][8];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (g4 + u >= gc) break;  // uniform over the warp
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                                 : "=r"(v[u][0]), "=r"(v[u][1]), "=r"(v[u][2]), "=r"(v[u][3]), "=r"(v[u][4]), "=r"(v[u][5]),
                                   "=r"(v[u][6]), "=r"(v[u][7])
                                 : "r"(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((g4 + u) * 32 + cb * 8)));
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int gi = g4 + u;
                    if (gi >= gc) break;
                    if constexpr (FMT == 16) {
#pragma unroll
                        for (int j = 0; j < 8; j++) av[j] += __uint_as_float(v[u][j]);
                    } else {
                        const uint2 sc = *reinterpret_cast<const uint2*>(wbuf + ((size_t)tt * gmax + gi) * CB +
                                                                         (FMT == 4 ? 512 : 1024) + (rr & 7) * 8);
                        const uint32_t sw = rr < 8 ? sc.x : sc.y;
                        const float sf = __uint_as_float(sw << 16), bf = __uint_as_float(sw & 0xffff0000u);
                        const float* ys = sYs + gi * BK_ROWS + cb * 8;
#pragma unroll
                        for (int j = 0; j < 8; j++) av[j] += sf * __uint_as_float(v[u][j]) + bf * ys[j];
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) sPart[m * BK_ROWS + cb * 8 + j] = av[j];
        }
        // the tensor memory goes back once every load above has completed
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncthreads();
        if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(tcols) : "memory");
    } else {
        // 4. warp w: tile w / wpt, groups w % wpt, + wpt, ...
        float acc[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        const int wpt = BK_WARPS / nt, t = warp / wpt;
        if (t < nt) {
            const uint32_t* xs = reinterpret_cast<const uint32_t*>(sX);
#pragma unroll 1
            for (int gi = warp - t * wpt; gi < gc; gi += wpt)
                bk_group<FMT>(wbuf + ((size_t)t * gmax + gi) * CB, xs + gi * 32, xs_b / 4, lo, ntl, sYs + gi * BK_ROWS, acc, lane);
        }
        __syncthreads();  // the staged rows are dead: their space takes the partial sums
        if (tr) tr[5] = gtimer();
        {
            const int g = lane >> 2, c = 2 * (lane & 3);
            float* r = sRed + warp * 16 * BK_ROWS;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                r[g * BK_ROWS + j * 8 + c] = acc[j][0];
                r[g * BK_ROWS + j * 8 + c + 1] = acc[j][1];
                r[(g + 8) * BK_ROWS + j * 8 + c] = acc[j][2];
                r[(g + 8) * BK_ROWS + j * 8 + c + 1] = acc[j][3];
            }
        }
        __syncthreads();
        // per tile: the sum of its warps, in warp order
        for (int e = tid; e < nt * 16 * BK_ROWS; e += BK_THREADS) {
            const int tt = e / (16 * BK_ROWS), rc = e - tt * 16 * BK_ROWS;
            float s = 0.f;
            for (int w = tt * wpt; w < (tt + 1) * wpt; w++) s += sRed[w * 16 * BK_ROWS + rc];
            sPart[e] = s;
        }
    }
    // 5. the ks ranks' partials (and x^2 sums), summed in rank order; rank r
    //    takes every ks-th (tile, row pair, activation row)
    cg::cluster_group cl = cg::this_cluster();
    if (ks > 1) cl.sync();
    else __syncthreads();
    if (tr) tr[6] = gtimer();
    for (int e = rank * BK_THREADS + tid; e < nt * 8 * BK_ROWS; e += ks * BK_THREADS) {
        const int tt = e / (8 * BK_ROWS), rem = e - tt * 8 * BK_ROWS, r8 = rem / BK_ROWS, col = rem - r8 * BK_ROWS;
        if (col >= nrows) continue;
        float lo = 0.f, hi = 0.f, ss = 0.f;
        for (int q = 0; q < ks; q++) {
            const float* pq = ks > 1 ? cl.map_shared_rank(sPart, q) : sPart;
            lo += pq[(tt * 16 + r8) * BK_ROWS + col];
            hi += pq[(tt * 16 + r8 + 8) * BK_ROWS + col];
            if (RMS) ss += (ks > 1 ? cl.map_shared_rank(sSS, q) : sSS)[col];
        }
        const float ps = RMS ? rsqrtf(ss / (float)W.K + in.eps) : 1.f;
        epi(tile0 + tt, r8, r0 + col, lo * ps, hi * ps);
    }
    // peers may still be reading this CTA's partials
    if (ks > 1) cl.sync();
    if (tr) tr[7] = gtimer();
}

// ---------------- host side ----------------

struct BulkPlan {
    int ks = 1, nb = 1, tmax = 1, gmax = 1, smem = 0;
};

// One CTA per SM: for each K split (1..8 ranks, a cluster) the tile ranges
// that fill the SMs, kept if a CTA holds at most 8 tiles and fits in shared
// memory; the cheapest by a latency model (per-warp mma groups, cluster
// rounds). (A 512-thread CTA holds most of an SM's registers, so the next
// kernel's CTAs start on an SM only as this kernel's leave it.)
inline BulkPlan bulk_plan_cap(int ntiles, int K, int rows, int fmt, int sms, bool lo, int cap, int ksmax) {
    const int ng = K / 64, cb = fmt == 4 ? 576 : (fmt == 8 ? 1088 : 2048);
    const int rb = (rows + BK_ROWS - 1) / BK_ROWS;
    BulkPlan best;
    long best_cost = -1;
    for (int ks = 1; ks <= ksmax && ks <= ng; ks++) {
        const int nb = std::min(ntiles, sms / (ks * rb));
        if (nb < 1) break;
        BulkPlan p;
        p.ks = ks;
        p.nb = nb;
        p.tmax = (ntiles + nb - 1) / nb;
        p.gmax = (ng + ks - 1) / ks;
        if (p.tmax > BK_TMAX) continue;
        p.smem = BulkSmem(p.tmax, p.gmax, cb, lo).total;
        if (p.smem > cap) continue;
        const int wpt = BK_WARPS / p.tmax;
        const long groups_per_warp = (p.gmax + wpt - 1) / wpt;
        const long cost = 3000 + 400L * groups_per_warp + 40L * p.gmax + 600L * (ks - 1);
        if (best_cost < 0 || cost < best_cost) {
            best = p;
            best_cost = cost;
        }
    }
    return best;
}

inline BulkPlan bulk_plan(int ntiles, int K, int rows, int fmt, int sms, bool lo, int ksmax) {
    return bulk_plan_cap(ntiles, K, rows, fmt, sms, lo, BK_SMEM_MAX, ksmax);
}

// tcgen05 plan: blocks of 8 tiles (128 features), K split so that a rank holds
// at most 16 groups (one 32-column accumulator each in 512 tensor-memory
// columns), one wave of CTAs; the cheapest by the same kind of latency model
// (a pipelined step per group, cluster rounds). smem 0 when none fits.
inline BulkPlan bulk_plan_tc(int ntiles, int K, int rows, int fmt, int sms, bool lo, bool force) {
    BulkPlan best;
    if (ntiles % 8) return best;
    const int ng = K / 64, cb = fmt == 4 ? 576 : (fmt == 8 ? 1088 : 2048), mb = ntiles / 8;
    const int rb = (rows + BK_ROWS - 1) / BK_ROWS;
    long best_cost = -1;
    for (int ks = std::max(1, (ng + 15) / 16); ks <= 8 && ks <= ng; ks++) {
        if ((long)mb * ks * rb > sms) break;
        if (!force && (long)mb * ks * rb * 2 < sms) continue;  // fewer than half the SMs: the mma.sync variant wins
        BulkPlan p;
        p.ks = ks;
        p.nb = mb;
        p.tmax = 8;
        p.gmax = (ng + ks - 1) / ks;
        if (p.gmax > 16) continue;
        p.smem = BulkSmem(8, p.gmax, cb, lo, true).total;
        if (p.smem > BK_SMEM_TC_MAX) continue;
        const long cost = 250L * p.gmax + (ks > 1 ? 800L + 100L * ks : 0L);
        if (best_cost < 0 || cost < best_cost) {
            best = p;
            best_cost = cost;
        }
    }
    return best;
}

// MING_BULK_TC=1 (read at each launch, so at graph capture) runs 4/8-bit
// weights in blocks of 128 features on the tcgen05 variant wherever a plan
// fits. Off by default: at this model's decode shapes the mma.sync variant is
// faster — the 128-feature blocks leave too few CTAs (gate/up: 76 for 148
// SMs) and each K group costs a staging round and a barrier. Measured per
// batch-32 step: 1.11 ms mma.sync; 1.25 ms with gate/up alone on tcgen05
// (4 stages, batched tensor-memory loads); 1.71 ms with every projection on
// it (2 stages, one load per group).
inline int bulk_tc_mode() {
    const char* v = getenv("MING_BULK_TC");
    return v && v[0] == '1' && v[1] == 0 ? 2 : 0;
}

template <int FMT, int PRO, bool TC, class Epi>
void launch_bulk_plan(const PackedW& W, const BulkIn& in, const Epi& e, int rows, const BulkPlan& p, cudaStream_t s) {
    static unsigned attr_devices = 0;  // bit d: attribute set on device d
    auto kern = linear_bulk_kernel<FMT, PRO, TC, Epi>;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_devices & (1u << (dev & 31)))) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TC ? BK_SMEM_TC_MAX : BK_SMEM_MAX);
        attr_devices |= 1u << (dev & 31);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.nb * p.ks), (unsigned)((rows + BK_ROWS - 1) / BK_ROWS));
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
    cudaLaunchKernelEx(&cfg, kern, W, in, e, rows, p.ks, p.nb, p.tmax, p.gmax);  // errors surface at the caller's check
}

// Launches the kernel; false when no plan fits (the caller takes another
// path).
template <int FMT, int PRO, class Epi>
bool launch_bulk(const PackedW& W, const BulkIn& in, const Epi& e, int rows, int sms, cudaStream_t s) {
    const bool lo = PRO == BK_RMS && in.nw;
    if constexpr (FMT != 16) {
        const int mode = bulk_tc_mode();
        if (PRO != BK_LNMOD && mode) {
            const BulkPlan p = bulk_plan_tc(W.ntiles, W.K, rows, FMT, sms, lo, mode == 2);
            if (p.smem) {
                launch_bulk_plan<FMT, PRO, true>(W, in, e, rows, p, s);
                return true;
            }
        }
    }
    const BulkPlan p = bulk_plan(W.ntiles, W.K, rows, FMT, sms, lo, PRO == BK_LNMOD ? 1 : 8);
    if (p.smem == 0) return false;
    launch_bulk_plan<FMT, PRO, false>(W, in, e, rows, p, s);
    return true;
}

}  // namespace ming
