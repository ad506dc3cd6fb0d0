// tcgen05.cuh — bf16 linears over many rows on the 5th-generation tensor
// cores (tcgen05.mma, accumulator in tensor memory).
//
// out[row][feature] = sum_k W[feature][k] * y[row][k] for bf16 weights and
// rows >= 64 (the DiT head at batch 32, prefill of a bf16 LM):
//   * a CTA owns 128 features (8 packed 16-row tiles, pack.h) and N rows
//     (64, 128 or 256); the f32 accumulator D[128][N] lives in tensor memory;
//   * both operands sit in global memory as the exact shared-memory image
//     the MMA reads — 128-byte-swizzled K-major blocks, one per 64-wide K
//     group: the weights are rewritten into 16 KB blocks once at load
//     (tc_swizzle_kernel), the activations by the stage kernel (prologue
//     once per value, stage_rows_kernel);
//   * a producer thread streams the two blocks of each K group with
//     cp.async.bulk into a 4-stage shared ring (full/empty mbarriers); an MMA
//     thread issues 4 tcgen05.mma (K = 16 each) per group and releases the
//     stage with tcgen05.commit; a last commit signals the epilogue;
//   * the epilogue reads D with tcgen05.ld (warp w: features 32 (w % 4) ..,
//     a quarter of the N rows per warp w / 4) and hands (tile, r8, row, lo,
//     hi) pairs to the same epilogue functors as the mma.sync kernels, every
//     lane busy (lanes r8 and r8 + 8 swap the halves of even/odd rows).
// Descriptor encodings follow the sm100 UMMA shared-memory and instruction
// descriptor layouts (CUTLASS 4, cute/arch/mma_sm100_desc.hpp).
#pragma once

#include <cooperative_groups.h>
#include <type_traits>

#include "linear.cuh"

namespace ming {

constexpr int TC_M = 128;  // features per CTA (tensor memory lanes)
constexpr int TC_THREADS = 512;  // 16 warps: the epilogue work of 128 x N outputs is spread over all of them
constexpr int TC_STAGES = 4;
constexpr int TC_A_BLOCK = TC_M * 128;  // bytes of one weight block (128 features x 64 bf16)

template <int N>
struct TcSmem {
    static constexpr int A_BYTES = TC_A_BLOCK;
    static constexpr int B_BYTES = N * 128;  // N rows x 64 bf16
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int TOTAL = 1024 + TC_STAGES * STAGE + 128;  // alignment slack, stages, barriers + tmem slot
    static constexpr int PART = TC_M * N * 4;                    // K split: this rank's f32 partial sums
    static constexpr int TOTAL_KS = TOTAL + PART;
};

// Byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled
// K-major block: 8-row atoms of 1024 bytes, chunk index XOR (row % 8).
MING_DEV uint32_t tc_sw128(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

// Shared-memory matrix descriptor: start address >> 4 at [0,14), leading
// byte offset (unused by swizzled K-major layouts) 1 at [16,30), stride byte
// offset 1024 >> 4 at [32,46), version 1 at [46,48), 128-byte swizzle (2) at
// [61,64).
MING_DEV uint64_t tc_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator (1 at [4,6)), A and B
// both bf16 (1 at [7,10) and [10,13)) or both f16 (0 there), both K-major,
// N >> 3 at [17,23), M >> 4 at [24,29).
template <int N, bool F16 = false>
MING_DEV constexpr uint32_t tc_idesc() {
    return (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(TC_M >> 4) << 24);
}

MING_DEV uint32_t tc_saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Bounded wait on an mbarrier phase (the waits here end in microseconds).
MING_DEV bool tc_mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t b = tc_saddr(bar);
    for (long long it = 0; it < (1ll << 26); it++) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(b), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

// Packed bf16 tiles -> swizzled weight blocks [ntiles / 8][K / 64][16 KB]:
// block (mt, g) is the shared-memory image of features 128 mt.. and K group g.
static __global__ void __launch_bounds__(TC_THREADS) tc_swizzle_kernel(const uint8_t* tiles, int ng, uint8_t* out) {
    const int mt = blockIdx.x, g = blockIdx.y;
    uint8_t* dst = out + ((size_t)mt * ng + g) * TC_A_BLOCK;
    for (int e = threadIdx.x; e < 8 * 4 * 32; e += TC_THREADS) {
        const int i = e >> 7, ks = (e >> 5) & 3, L = e & 31;
        const uint4 w = *reinterpret_cast<const uint4*>(tiles + ((size_t)(mt * 8 + i) * ng + g) * 2048 + ((size_t)ks * 32 + L) * 16);
        // the lane's mma.sync A fragment: (row g, k), (row g+8, k), (row g, k+8), (row g+8, k+8), k = 16 ks + 2 (L % 4)
        const int r0 = i * 16 + (L >> 2), k0 = ks * 16 + 2 * (L & 3);
        const int c0 = k0 >> 3, b0 = (2 * k0) & 15;
        *reinterpret_cast<uint32_t*>(dst + tc_sw128(r0, c0) + b0) = w.x;
        *reinterpret_cast<uint32_t*>(dst + tc_sw128(r0 + 8, c0) + b0) = w.y;
        *reinterpret_cast<uint32_t*>(dst + tc_sw128(r0, c0 + 1) + b0) = w.z;
        *reinterpret_cast<uint32_t*>(dst + tc_sw128(r0 + 8, c0 + 1) + b0) = w.w;
    }
}

// Packed 4/8-bit tiles -> swizzled f16 weight blocks over twice the K groups:
// each weight dequantized as MLX's affine dequantize does (w = scale * q +
// bias in f32) and split into hi = f16(w) (group g) and lo = f16(w - hi)
// (group ng + g), so that the tcgen05 sums over the rows staged twice keep
// ~22 significant bits of every weight: the prefill copy of a quantized
// linear, as accurate as the exact-weight mma.sync kernels.
static __global__ void __launch_bounds__(TC_THREADS) tc_swizzle_dq_kernel(const uint8_t* tiles, int ng, int fmt, uint8_t* out) {
    const int mt = blockIdx.x, g = blockIdx.y, cb = fmt == 4 ? 576 : 1088;
    uint8_t* dhi = out + ((size_t)mt * 2 * ng + g) * TC_A_BLOCK;
    uint8_t* dlo = dhi + (size_t)ng * TC_A_BLOCK;
    for (int e = threadIdx.x; e < 8 * 4 * 32; e += TC_THREADS) {
        const int i = e >> 7, ks = (e >> 5) & 3, L = e & 31;
        const uint8_t* ch = tiles + ((size_t)(mt * 8 + i) * ng + g) * cb;
        const uint2 sc = *reinterpret_cast<const uint2*>(ch + (fmt == 4 ? 512 : 1024) + (L >> 2) * 8);
        const float s_lo = __uint_as_float(sc.x << 16), b_lo = __uint_as_float(sc.x & 0xffff0000u);
        const float s_hi = __uint_as_float(sc.y << 16), b_hi = __uint_as_float(sc.y & 0xffff0000u);
        uint32_t q[4];
        if (fmt == 4) {
            dq4(reinterpret_cast<const uint32_t*>(ch + (size_t)L * 16)[ks], q);
        } else {
            const uint32_t* w8 = reinterpret_cast<const uint32_t*>(ch + ((size_t)(ks >> 1) * 32 + L) * 16 + (ks & 1) * 8);
            dq8(w8[0], w8[1], q);
        }
        // q[0..3]: (row r, k..k+1), (row r+8, k..), (row r, k+8..), (row r+8, k+8..) as exact f16 codes
        uint32_t wh[4], wl[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&q[j]));
            const float sj = (j & 1) ? s_hi : s_lo, bj = (j & 1) ? b_hi : b_lo;
            const float w0 = sj * v.x + bj, w1 = sj * v.y + bj;
            wh[j] = pack_f16x2(w0, w1);
            const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&wh[j]));
            wl[j] = pack_f16x2(w0 - h.x, w1 - h.y);
        }
        const int r0 = i * 16 + (L >> 2), k0 = ks * 16 + 2 * (L & 3);
        const int c0 = k0 >> 3, b0 = (2 * k0) & 15;
        const uint32_t o[4] = {tc_sw128(r0, c0) + b0, tc_sw128(r0 + 8, c0) + b0, tc_sw128(r0, c0 + 1) + b0,
                               tc_sw128(r0 + 8, c0 + 1) + b0};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            *reinterpret_cast<uint32_t*>(dhi + o[j]) = wh[j];
            *reinterpret_cast<uint32_t*>(dlo + o[j]) = wl[j];
        }
    }
}

// The rows of a prologue over two K sections (the hi and lo weight blocks of
// a split prefill copy): y(row, k) = pro.y(row, k mod K).
template <class Pro>
struct ProTwice {
    Pro p;
    int K;
    MING_DEV void init(int r0, int nrows, float* aux) { p.init(r0, nrows, aux); }
    MING_DEV float y(int row, int k) const { return p.y(row, k < K ? k : k - K); }
    MING_DEV float post(int row) const { return p.post(row); }
};

// Rows -> swizzled activation blocks [rows / N][K / 64][N * 128 bytes]: the
// prologue once per (row, k), with the operand rounding of the mma.sync
// kernels (pack_bf16x2), and each row's post scale. Rows past `rows` in the
// last block are left as they are (their outputs are never written).
template <int N, class Pro, bool F16 = false>
__global__ void __launch_bounds__(LIN_THREADS) stage_rows_kernel(Pro pro, int rows, int K, uint8_t* xs, float* post) {
    __shared__ float aux[8 * 32];
    const int r0 = blockIdx.x * 8, nrows = min(8, rows - r0);
    const int kc = blockIdx.y * STAGE_KC, kcl = min(STAGE_KC, K - kc), ng = K / 64;
    // the rows are the previous kernel's output; the linear that reads this
    // kernel's blocks may launch and fetch its weights meanwhile
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    Pro p = pro;
    p.init(r0, nrows, aux);
    __syncthreads();
    // one 16-byte swizzled chunk (8 consecutive k of a row) per item: the 8
    // prologue values are independent, then one store
    bool vec = false;  // the prologue's 16-byte path (ProPlain, ProLnMod) when the layout allows it
    if constexpr (std::is_same_v<Pro, ProPlain>) vec = p.ld % 8 == 0 && ((uintptr_t)p.x & 15) == 0;
    else if constexpr (std::is_same_v<Pro, ProLnMod>) vec = p.y8_ok();
    for (int e = threadIdx.x; e < nrows * (kcl / 8); e += LIN_THREADS) {
        const int row = e / (kcl / 8), k = kc + 8 * (e % (kcl / 8)), n = r0 + row;
        float y[8];
        if constexpr (std::is_same_v<Pro, ProPlain> || std::is_same_v<Pro, ProLnMod>) {
            if (vec) p.y8(row, k, y);
            else {
#pragma unroll
                for (int u = 0; u < 8; u++) y[u] = p.y(row, k + u);
            }
        } else {
#pragma unroll
            for (int u = 0; u < 8; u++) y[u] = p.y(row, k + u);
        }
        uint8_t* blk = xs + ((size_t)(n / N) * ng + k / 64) * (N * 128);
        if constexpr (F16)
            *reinterpret_cast<uint4*>(blk + tc_sw128(n % N, (k & 63) >> 3)) =
                make_uint4(pack_f16x2(y[0], y[1]), pack_f16x2(y[2], y[3]), pack_f16x2(y[4], y[5]), pack_f16x2(y[6], y[7]));
        else
            *reinterpret_cast<uint4*>(blk + tc_sw128(n % N, (k & 63) >> 3)) =
                make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
    }
    if (blockIdx.y == 0 && threadIdx.x < nrows) post[r0 + threadIdx.x] = p.post(threadIdx.x);
}

// Grid: x = block of 8 packed tiles (128 features) * nks + K rank, y = block
// of N rows. nks > 1: the K groups are split over a thread-block cluster of
// nks CTAs; each rank's accumulator goes to shared memory and the ranks' sums
// meet over distributed shared memory in rank order (deterministic), the
// ranks splitting the epilogue.
// Thread 0 produces, thread 32 issues the MMAs, all 16 warps run the epilogue.
template <int N, class Epi, bool F16 = false>
__global__ void __launch_bounds__(TC_THREADS) tc_linear_kernel(const uint8_t* wtc, int K, const uint8_t* xs, const float* post,
                                                               Epi epi, int rows, int nks) {
    using S = TcSmem<N>;
    extern __shared__ __align__(16) uint8_t tc_smem_raw[];
    // 1024-byte aligned base: the swizzle atoms are anchored at 1024 bytes
    const uint32_t raw = tc_saddr(tc_smem_raw);
    uint8_t* smem = tc_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + TC_STAGES * S::STAGE);  // [TC_STAGES]
    uint64_t* empty = full + TC_STAGES;                                          // [TC_STAGES]
    uint64_t* done = empty + TC_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    float* part = reinterpret_cast<float*>(smem + S::TOTAL - 1024);  // nks > 1: [128 features][N rows]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x / nks, rank = blockIdx.x % nks, nt = blockIdx.y, n0 = nt * N, ngt = K / 64;
    // this rank's K groups [gb, gb + ng)
    const int gb = rank * ngt / nks, ng = (rank + 1) * ngt / nks - gb;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tc_saddr(tmem_slot)), "r"(N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < TC_STAGES; s++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_saddr(&full[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_saddr(&empty[s])));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_saddr(done)));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    // warp 0 lane 0 produces, warp 1 lane 0 issues the MMAs; the other lanes of
    // those warps park at __syncwarp instead of spinning beside them
    if (tid == 0) {
        // producer: the weight block and the activation block of each K group.
        // The first stages' weight blocks go out before the wait on the
        // previous kernel (the launch is its programmatic dependent; weights
        // do not depend on it), their activation blocks after it.
        const uint8_t* wa = wtc + ((size_t)mt * ngt + gb) * S::A_BYTES;
        const uint8_t* xb = xs + ((size_t)nt * ngt + gb) * S::B_BYTES;
        const int pre = ng < TC_STAGES ? ng : TC_STAGES;
        for (int g = 0; g < pre; g++) {
            uint8_t* sA = smem + g * S::STAGE;
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(tc_saddr(&full[g])),
                         "r"((uint32_t)S::STAGE)
                         : "memory");
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                             tc_saddr(sA)),
                         "l"(wa + (size_t)g * S::A_BYTES), "r"((uint32_t)S::A_BYTES), "r"(tc_saddr(&full[g]))
                         : "memory");
        }
        asm volatile("griddepcontrol.wait;\n" ::: "memory");
        for (int g = 0; g < ng; g++) {
            const int s = g % TC_STAGES;
            uint8_t* sA = smem + s * S::STAGE;
            if (g >= pre) {
                if (!tc_mbar_wait(&empty[s], ((g / TC_STAGES) - 1) & 1)) break;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(tc_saddr(&full[s])),
                             "r"((uint32_t)S::STAGE)
                             : "memory");
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                                 tc_saddr(sA)),
                             "l"(wa + (size_t)g * S::A_BYTES), "r"((uint32_t)S::A_BYTES), "r"(tc_saddr(&full[s]))
                             : "memory");
            }
            asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                             tc_saddr(sA + S::A_BYTES)),
                         "l"(xb + (size_t)g * S::B_BYTES), "r"((uint32_t)S::B_BYTES), "r"(tc_saddr(&full[s]))
                         : "memory");
        }
    } else if (tid == 32) {
        // MMA issuer
        int g = 0;
        for (; g < ng; g++) {
            const int s = g % TC_STAGES;
            if (!tc_mbar_wait(&full[s], (g / TC_STAGES) & 1)) break;
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t a0 = tc_saddr(smem + s * S::STAGE), b0 = a0 + S::A_BYTES;
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                const uint64_t da = tc_desc(a0 + 32 * ks), db = tc_desc(b0 + 32 * ks);
                const uint32_t acc = (g > 0 || ks > 0) ? 1u : 0u;
                asm volatile(
                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                    " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                    "l"(da), "l"(db), "r"(tc_idesc<N, F16>()), "r"(acc)
                    : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                             tc_saddr(&empty[s]))
                         : "memory");
        }
        // every MMA issued (all, unless a wait gave up) completes before this arrives
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(tc_saddr(done))
                     : "memory");
    }
    if (warp < 2) __syncwarp();
    // the epilogue reads the row scales and residuals the previous kernels wrote
    if (tid != 0) asm volatile("griddepcontrol.wait;\n" ::: "memory");
    const bool ok = tc_mbar_wait(done, 0);
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    // epilogue: warp w reads features m = 32 (w % 4) + lane (its tensor-memory
    // lane quarter) for rows [q N / 4, (q + 1) N / 4), q = w / 4. Feature pairs
    // (r8, r8 + 8) of a tile sit on lanes 8 apart: the lane holding r8 takes
    // the even rows, its partner the odd ones, each getting the other half by
    // one shuffle.
    const int quarter = warp & 3, m = quarter * 32 + lane, hi_lane = lane & 8;
    const int cbeg = (warp >> 2) * (N / 4), cend = cbeg + N / 4;
    if (nks > 1) {
        // this rank's partial sums -> shared memory [m][n]
        for (int c0 = cbeg; c0 < cend; c0 += 16) {
            uint32_t v[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
                  "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                : "r"(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0));
            asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
            for (int j = 0; j < 16; j++) part[m * N + c0 + j] = __uint_as_float(v[j]);
        }
        // tensor memory back before the cluster barrier (ranks on one SM never wait on each other's columns)
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncthreads();
        if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(N) : "memory");
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        // rank r: every ks-th (tile, tile row r8, row n); the ranks' sums in rank order
        for (int e = rank * TC_THREADS + tid; e < 8 * 8 * N; e += nks * TC_THREADS) {
            const int t = e / (8 * N), rem = e - t * 8 * N, r8 = rem / N, n = rem - r8 * N;
            if (n0 + n >= rows) continue;
            float lo = 0.f, hi = 0.f;
            for (int q = 0; q < nks; q++) {
                const float* pq = cl.map_shared_rank(part, q);
                lo += pq[(t * 16 + r8) * N + n];
                hi += pq[(t * 16 + r8 + 8) * N + n];
            }
            if (ok) {
                const float ps = post[n0 + n];
                epi(mt * 8 + t, r8, n0 + n, lo * ps, hi * ps);
            }
        }
        cl.sync();  // peers may still be reading this CTA's partials
        return;
    }
    for (int c0 = cbeg; c0 < cend; c0 += 16) {
        uint32_t v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
              "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
            const float ev = __uint_as_float(v[2 * jj]), od = __uint_as_float(v[2 * jj + 1]);
            const float other = __shfl_xor_sync(0xffffffffu, hi_lane ? ev : od, 8);
            const float lo = hi_lane ? other : ev, hi = hi_lane ? od : other;
            const int n = n0 + c0 + 2 * jj + (hi_lane ? 1 : 0);
            if (n < rows && ok) {
                const float ps = post[n];
                epi(mt * 8 + (m >> 4), lane & 7, n, lo * ps, hi * ps);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(N) : "memory");
}

}  // namespace ming
