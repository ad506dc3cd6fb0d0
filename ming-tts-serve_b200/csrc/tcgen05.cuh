// tcgen05.cuh — bf16 linears over many rows on the 5th-generation tensor
// cores (tcgen05.mma, accumulator in tensor memory).
//
// out[row][feature] = sum_k W[feature][k] * y[row][k] for bf16 weights and
// rows >= 64 (the DiT head at batch 32, prefill of a bf16 LM):
//   * a CTA owns 128 features (8 packed 16-row tiles, pack.h) and N rows
//     (64, 128 or 256); the f32 accumulator D[128][N] lives in tensor memory;
//   * per 64-wide K group the CTA's threads rewrite the 8 packed tile chunks
//     (mma.sync fragment order) into a 128-byte-swizzled K-major shared tile
//     and copy the N activation rows (the prologue's output, staged once,
//     row-major bf16) with cp.async into the same swizzled layout;
//   * one thread issues 4 tcgen05.mma (K = 16 each) and commits them to the
//     stage's mbarrier; two stages let the copies of group g+1 overlap the
//     MMAs of group g;
//   * the epilogue reads D with tcgen05.ld (warp w: features 32w..32w+31)
//     and hands (tile, r8, row, lo, hi) pairs to the same epilogue functors
//     as the mma.sync kernels.
// Descriptor encodings follow the sm100 UMMA shared-memory and instruction
// descriptor layouts (CUTLASS 4, cute/arch/mma_sm100_desc.hpp).
#pragma once

#include "linear.cuh"

namespace ming {

constexpr int TC_M = 128;  // features per CTA (tensor memory lanes)
constexpr int TC_THREADS = 128;

template <int N>
struct TcSmem {
    static constexpr int A_BYTES = TC_M * 128;  // 128 features x 64 bf16
    static constexpr int B_BYTES = N * 128;     // N rows x 64 bf16
    static constexpr int STAGE = A_BYTES + B_BYTES;
    static constexpr int TOTAL = 1024 + 2 * STAGE + 64;  // alignment slack, 2 stages, barriers + tmem slot
};

// Byte offset of 16-byte chunk c (0..7) of row r in a 128-byte-swizzled
// K-major tile: 8-row atoms of 1024 bytes, chunk index XOR (row % 8).
MING_DEV uint32_t tc_sw128(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

// Shared-memory matrix descriptor: start address >> 4 at [0,14), leading
// byte offset (unused by swizzled K-major layouts) 1 at [16,30), stride byte
// offset 1024 >> 4 at [32,46), version 1 at [46,48), 128-byte swizzle (2) at
// [61,64).
MING_DEV uint64_t tc_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator (1 at [4,6)), bf16 A and
// B (1 at [7,10) and [10,13)), both K-major, N >> 3 at [17,23), M >> 4 at [24,29).
template <int N>
MING_DEV constexpr uint32_t tc_idesc() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);
}

MING_DEV uint32_t tc_saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MING_DEV bool tc_mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t b = tc_saddr(bar);
    for (long long it = 0; it < (1ll << 26); it++) {  // bounded: the tensor cores finish in microseconds
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

// Rows -> row-major bf16 activations: the prologue once per (row, k), with
// the operand rounding of the mma.sync kernels (pack_bf16x2), and each row's
// post scale.
template <class Pro>
__global__ void __launch_bounds__(LIN_THREADS) stage_rows_kernel(Pro pro, int rows, int K, uint16_t* xs, float* post) {
    __shared__ float aux[8 * 32];
    const int r0 = blockIdx.x * 8, nrows = min(8, rows - r0);
    const int kc = blockIdx.y * STAGE_KC, kcl = min(STAGE_KC, K - kc);
    Pro p = pro;
    p.init(r0, nrows, aux);
    __syncthreads();
    for (int e = threadIdx.x; e < nrows * (kcl / 2); e += LIN_THREADS) {
        const int row = e / (kcl / 2), k = kc + 2 * (e % (kcl / 2));
        *reinterpret_cast<uint32_t*>(xs + (size_t)(r0 + row) * K + k) = pack_bf16x2(p.y(row, k), p.y(row, k + 1));
    }
    if (blockIdx.y == 0 && threadIdx.x < nrows) post[r0 + threadIdx.x] = p.post(threadIdx.x);
}

// Grid: x = block of 8 packed tiles (128 features), y = block of N rows.
template <int N, class Epi>
__global__ void __launch_bounds__(TC_THREADS) tc_linear_kernel(PackedW W, const uint16_t* xs, const float* post, Epi epi,
                                                               int rows) {
    using S = TcSmem<N>;
    extern __shared__ __align__(16) uint8_t tc_smem_raw[];
    // 1024-byte aligned base: the swizzle atoms are anchored at 1024 bytes
    const uint32_t raw = tc_saddr(tc_smem_raw);
    uint8_t* smem = tc_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + 2 * S::STAGE);  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mbar + 2);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mt = blockIdx.x, n0 = blockIdx.y * N, ng = W.K / 64;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tc_saddr(tmem_slot)), "r"(N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_saddr(&mbar[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_saddr(&mbar[1])));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    for (int g = 0; g < ng; g++) {
        const int st = g & 1;
        uint8_t* sA = smem + st * S::STAGE;
        uint8_t* sB = sA + S::A_BYTES;
        if (g >= 2) ok &= tc_mbar_wait(&mbar[st], ((g - 2) >> 1) & 1);  // the MMAs that read this stage are done
        // weights: 8 tiles x 4 k-steps x 32 lanes of 16-byte fragment words
        for (int e = tid; e < 8 * 4 * 32; e += TC_THREADS) {
            const int i = e >> 7, ks = (e >> 5) & 3, L = e & 31;
            const uint4 w = ldg_nc16(W.tiles + ((size_t)(mt * 8 + i) * ng + g) * 2048 + ((size_t)ks * 32 + L) * 16);
            const int r0 = i * 16 + (L >> 2), k0 = ks * 16 + 2 * (L & 3);  // element (r0, k0..k0+1) and friends
            const int c0 = k0 >> 3, b0 = (2 * k0) & 15;
            *reinterpret_cast<uint32_t*>(sA + tc_sw128(r0, c0) + b0) = w.x;
            *reinterpret_cast<uint32_t*>(sA + tc_sw128(r0 + 8, c0) + b0) = w.y;
            *reinterpret_cast<uint32_t*>(sA + tc_sw128(r0, c0 + 1) + b0) = w.z;
            *reinterpret_cast<uint32_t*>(sA + tc_sw128(r0 + 8, c0 + 1) + b0) = w.w;
        }
        // activations: N rows x 8 chunks of 16 bytes
        for (int e = tid; e < N * 8; e += TC_THREADS) {
            const int n = e >> 3, c = e & 7;
            uint8_t* dst = sB + tc_sw128(n, c);
            if (n0 + n < rows) {
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(tc_saddr(dst)),
                             "l"(xs + (size_t)(n0 + n) * W.K + g * 64 + c * 8)
                             : "memory");
            } else {
                *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
            }
        }
        asm volatile("cp.async.wait_all;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic-proxy writes -> tensor-core reads
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t a0 = tc_saddr(sA), b0 = tc_saddr(sB);
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                const uint64_t da = tc_desc(a0 + 32 * ks), db = tc_desc(b0 + 32 * ks);
                const uint32_t acc = (g > 0 || ks > 0) ? 1u : 0u;
                asm volatile(
                    "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                    " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
                    "l"(da), "l"(db), "r"(tc_idesc<N>()), "r"(acc)
                    : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                             tc_saddr(&mbar[st]))
                         : "memory");
        }
    }
    ok &= tc_mbar_wait(&mbar[(ng - 1) & 1], ((ng - 1) >> 1) & 1);  // every MMA of the CTA has completed
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    // epilogue: warp w reads features 32w + lane; row pairs (r8, r8 + 8) of a tile are lanes 8 apart
    const int m = warp * 32 + lane;
    for (int c0 = 0; c0 < N; c0 += 16) {
        uint32_t v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
              "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const float lo = __uint_as_float(v[j]);
            const float hi = __shfl_down_sync(0xffffffffu, lo, 8);
            const int n = n0 + c0 + j;
            if ((lane & 15) < 8 && n < rows && ok) {
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
