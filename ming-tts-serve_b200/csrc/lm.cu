// lm.cu — paged split-K decode attention, final norm + stop head, step
// bookkeeping kernels.
#include <cuda_runtime.h>

#include <cooperative_groups.h>

#include "lm.cuh"

namespace ming {

// One CTA per (split, kv head, row). Scores of the 7 query heads sharing the kv
// head against the split's positions (two-pass softmax inside the split, as
// the reference's LB kernel, src/ming_fused.zig:326-374), then P.V.
// Partial (m, l, acc) go to `part` for the O prologue to combine.
namespace {
constexpr int ATT_MAXG = 8;     // query heads per kv head (<= 8)
constexpr int ATT_KS = HD + 8;  // padded q row (elements) of the mma A operand
constexpr int ATT_ROWB = HD * 2;                       // K/V row in shared memory: 128 B, as a page stores it
constexpr int ATT_KV = ATT_SPLIT * ATT_ROWB;           // one split's K (or V) rows
constexpr int ATT_BODY = 2 * ATT_KV + ATT_MAXG * HD * 4 + ATT_MAXG * ATT_SPLIT * 4;
constexpr int ATT_SMEM = 1024 + ATT_BODY + 16;         // 1024-byte alignment slack (128-byte swizzle) + mbarrier
constexpr int ATT_SMEM_CL = ATT_SMEM + ATT_MAXG * PART_STRIDE * 4;
constexpr long long ATT_TIMEOUT = 4000000000LL;        // cycles (~2 s) before a page-copy wait gives up
static_assert(8 * ATT_MAXG * 32 * 8 <= ATT_KV, "P.V partial sums fit in the key area");
static_assert(8 * ATT_MAXG * PART_STRIDE * 4 <= ATT_KV && (ATT_MAXG * PART_STRIDE) % 4 == 0,
              "eight ranks' partials fit in the key area as float4");

MING_DEV uint32_t att_su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// Element offset of (row, dim) in a 128-byte-swizzled K/V block: 16-byte
// chunk c of row r sits at chunk c ^ (r % 8) (the TMA's SWIZZLE_128B on a
// 1024-byte-aligned block).
MING_DEV int att_sw(int r, int d) { return r * HD + ((((d >> 3) ^ (r & 7))) << 3) + (d & 7); }
MING_DEV bool att_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(att_su32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
MING_DEV bool att_wait(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!att_try(bar, parity))
        if (clock64() - t0 > ATT_TIMEOUT) return false;
    return true;
}
// One 16-row page of K or V (2 KB) by TMA into a 1024-byte-aligned slot
MING_DEV void att_page(void* dst, const CUtensorMap* m, int row0, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
            att_su32(dst)),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(0), "r"(row0), "r"(att_su32(bar))
        : "memory");
}
}  // namespace

bool make_kv_tensor_map(CUtensorMap* m, uint16_t* pool, long long rows) {
    using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
        q != cudaDriverEntryPointSuccess)
        return false;
    const cuuint64_t dims[2] = {(cuuint64_t)HD, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)HD * 2};
    const cuuint32_t box[2] = {(cuuint32_t)HD, (cuuint32_t)PAGE};
    const cuuint32_t estr[2] = {1, 1};
    return reinterpret_cast<Encode>(fn)(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, pool, dims, strides, box, estr,
                                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// One (split, kv head, row): the row's causal positions [p0, p1) of one
// 256-position split, every query head of the kv group. The split's K and V
// pages (16 positions x 128 B each) come in by TMA, one tiled copy per page on
// one mbarrier, landing 128-byte-swizzled so that the mma fragment reads and
// the ldmatrix rows hit 32 distinct banks. Then scores on the tensor cores
// (mma.sync, the group's heads as the 16-row A operand), a per-head softmax
// inside the split in f32, and P.V on the tensor cores (a warp per 8 dims, P
// as bf16 hi + lo parts).
// CL = false: (max, sum, unnormalised P.V) per head go to `part`, combined by
// attn_combine_kernel. CL = true: the splits of one (kv head, row) are one
// thread-block cluster; each keeps its partials in shared memory, copies
// every rank's partials over distributed shared memory after a cluster
// barrier, and rank r combines heads r, r + ns, ... (the combine kernel's
// formula and split order) into `att`.
// A page copy that never lands (bounded wait) sets ATT_ERR_PAGES in a.err; the
// CTA then skips its compute, still takes the cluster barriers, and waits
// (bounded again) for its copies before it exits.
template <bool CL>
__global__ void __launch_bounds__(256, 2) attn_partial_kernel(const AttnArgs a, const __grid_constant__ CUtensorMap tmap) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (att_su32(smem_raw) & 1023u)) & 1023u);
    uint16_t* sK = reinterpret_cast<uint16_t*>(smem);                          // [ATT_SPLIT][HD], swizzled
    uint16_t* sV = reinterpret_cast<uint16_t*>(smem + ATT_KV);                 // [ATT_SPLIT][HD], swizzled
    float* sq = reinterpret_cast<float*>(smem + 2 * ATT_KV);                   // [ATT_MAXG][HD]
    float* sc = sq + ATT_MAXG * HD;                                            // [ATT_MAXG][ATT_SPLIT]
    uint64_t* bar = reinterpret_cast<uint64_t*>(sc + ATT_MAXG * ATT_SPLIT);   // the pages' mbarrier
    float* sO = reinterpret_cast<float*>(bar + 2);                             // CL: [ATT_MAXG][PART_STRIDE]
    uint16_t* sQ = reinterpret_cast<uint16_t*>(sq);                            // q as bf16: [ATT_MAXG][ATT_KS]
    const int split = blockIdx.x, kh = blockIdx.y, row = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = a.heads / a.kv_heads;
    const int pos = a.rows.pos[row], seq = a.rows.seq[row];
    const int n = pos + 1, p0 = split * ATT_SPLIT, p1 = min(n, p0 + ATT_SPLIT), len = p1 - p0;
    const bool live = p0 < n;  // CTA-uniform
    long long* tr =
        a.trace && tid == 0 ? a.trace + (((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x) * 8 : nullptr;
    if (tr) tr[0] = gtimer();
    float* out = CL ? sO : a.part + ((size_t)row * a.nsplit_max + split) * a.heads * PART_STRIDE + (size_t)kh * grp * PART_STRIDE;
    if (!CL && !live) return;  // split unused for this row (never read by the combine)
    const int* bt = a.kv.bt + (size_t)seq * a.kv.bt_ld;
    const int np = (len + PAGE - 1) / PAGE;  // pages of the split (p0 is page-aligned)
    // page i of the split: its K (which = 0) or V (1) rows in the pool as rows of the tensor map
    auto page_row = [&](int i, int which) {
        return (((bt[p0 / PAGE + i] * a.kv.layers + a.layer) * 2 + which) * a.kv.kv_heads + kh) * PAGE;
    };
    auto fetch = [&](int ia, int ib) {
        for (int i = ia; i < ib; i++) {
            att_page(sK + i * PAGE * HD, &tmap, page_row(i, 0), bar);
            att_page(sV + i * PAGE * HD, &tmap, page_row(i, 1), bar);
        }
    };
    // Decode: pages wholly before the row's own position were cached by
    // earlier steps and are fetched before the wait on the q|k|v kernel
    // (launched with programmatic stream serialization); the rest after it.
    const int pre = live && a.decode ? max(0, min(np, pos / PAGE - p0 / PAGE)) : 0;
    if (live && tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(att_su32(bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(att_su32(bar)),
                     "r"(np * 2 * PAGE * HD * 2)
                     : "memory");
        fetch(0, pre);
    }
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (tr) tr[1] = gtimer();
    bool failed = false;
    if (live) {
        if (tid == 0) fetch(pre, np);
        // q of the group's heads as bf16 (the mma A operand; heads >= grp are
        // zero rows); the 1/8 scale is applied to the f32 sums
        for (int e = tid; e < ATT_MAXG * HD; e += 256) {
            const int i = e / HD, d = e % HD;
            sQ[i * ATT_KS + d] = i < grp ? a.q[(size_t)row * a.heads * HD + (kh * grp + i) * HD + d] : (uint16_t)0;
        }
        __syncthreads();  // the barrier's initialisation is visible to every thread
        failed = __syncthreads_or(!att_wait(bar, 0));
    }
    if (failed) {
        if (tid == 0) {
            if (a.err) atomicCAS(a.err, 0, ATT_ERR_PAGES);
            att_wait(bar, 0);  // the copies in flight land before the CTA's shared memory is released
        }
        // an empty partial (weight 0) in place of this split's
        for (int e = tid; e < grp * PART_STRIDE; e += 256) out[e] = e % PART_STRIDE == 0 ? -INFINITY : 0.f;
    } else if (live) {
        // V rows from len up to the next 16-position k-step are read by the
        // last P.V k-step with P = 0: make them finite (whole rows, so the
        // swizzle does not matter)
        for (int e = tid; e < (((len + 15) & ~15) - len) * (HD / 2); e += 256) {
            const int j = len + e / (HD / 2), d2 = e % (HD / 2);
            *reinterpret_cast<uint32_t*>(sV + j * HD + 2 * d2) = 0u;
        }
        __syncthreads();
        if (tr) tr[2] = gtimer();
        const int g = lane >> 2, t4 = lane & 3;
        {
            // scores S = Q K^T on the tensor cores: rows = query heads (8 of
            // the 16 used), 8-position n-tiles strided over the warps, 4
            // k-steps of 16 dims; key columns past len are computed and
            // dropped (each output column reads only its own key row)
            uint32_t qa[4][2];
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                qa[ks][0] = *reinterpret_cast<const uint32_t*>(sQ + g * ATT_KS + ks * 16 + 2 * t4);
                qa[ks][1] = *reinterpret_cast<const uint32_t*>(sQ + g * ATT_KS + ks * 16 + 8 + 2 * t4);
            }
            const int nte = (len + 7) >> 3;
            for (int nt = warp; nt < nte; nt += 8) {
                float c[4] = {0.f, 0.f, 0.f, 0.f};
                const int R = nt * 8 + g;
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    const uint32_t af[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
                    mma_bf16(c, af, *reinterpret_cast<const uint32_t*>(sK + att_sw(R, ks * 16 + 2 * t4)),
                             *reinterpret_cast<const uint32_t*>(sK + att_sw(R, ks * 16 + 8 + 2 * t4)));
                }
                const int j = nt * 8 + 2 * t4;
                if (g < grp) {
                    if (j < len) sc[g * ATT_SPLIT + j] = 0.125f * c[0];
                    if (j + 1 < len) sc[g * ATT_SPLIT + j + 1] = 0.125f * c[1];
                }
            }
        }
        __syncthreads();
        if (tr) tr[3] = gtimer();
        if (warp < grp) {
            float m = -INFINITY;
            for (int j = lane; j < len; j += 32) m = fmaxf(m, sc[warp * ATT_SPLIT + j]);
            m = warp_max(m);
            float l = 0.f;
            for (int j = lane; j < len; j += 32) {
                const float p = expf(sc[warp * ATT_SPLIT + j] - m);
                sc[warp * ATT_SPLIT + j] = p;
                l += p;
            }
            l = warp_sum(l);
            if (lane == 0) {
                float* o = out + (size_t)warp * PART_STRIDE;
                o[0] = m;
                o[1] = l;
            }
        }
        __syncthreads();
        if (tr) tr[4] = gtimer();
        {
            // P.V on the tensor cores: warp w owns dims [8w, 8w + 8) over all
            // 16-position k-steps. P (f32) enters as bf16 hi + lo parts (two
            // mma on the same V fragment, ~2^-16 relative), V fragments come
            // from the row-major rows with ldmatrix.trans; positions past len
            // have P = 0
            const int n0 = warp * 8, kte = (len + 15) >> 4;
            const float* pr = sc + (g < grp ? g : 0) * ATT_SPLIT;
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            for (int kt = 0; kt < kte; kt++) {
                const int j = kt * 16 + 2 * t4;
                float2 pa, pb;
                if (j + 9 < len) {
                    pa = *reinterpret_cast<const float2*>(pr + j);
                    pb = *reinterpret_cast<const float2*>(pr + j + 8);
                } else {
                    pa = make_float2(j < len ? pr[j] : 0.f, j + 1 < len ? pr[j + 1] : 0.f);
                    pb = make_float2(j + 8 < len ? pr[j + 8] : 0.f, j + 9 < len ? pr[j + 9] : 0.f);
                }
                const float ha = rb(pa.x), hb = rb(pa.y), hc = rb(pb.x), hd = rb(pb.y);
                const uint32_t ah[4] = {pack_bf16x2(ha, hb), 0u, pack_bf16x2(hc, hd), 0u};
                const uint32_t al[4] = {pack_bf16x2(pa.x - ha, pa.y - hb), 0u, pack_bf16x2(pb.x - hc, pb.y - hd), 0u};
                uint32_t b0, b1;
                const uint16_t* vr = sV + att_sw(kt * 16 + (lane & 15), n0);
                asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];\n"
                             : "=r"(b0), "=r"(b1)
                             : "r"(att_su32(vr)));
                mma_bf16(c, ah, b0, b1);
                mma_bf16(c, al, b0, b1);
            }
            if (g < grp) {
                float* ob = out + (size_t)g * PART_STRIDE;
                ob[2 + n0 + 2 * t4] = c[0];
                ob[3 + n0 + 2 * t4] = c[1];
            }
        }
        if (tr) tr[5] = gtimer();
    } else if (CL) {
        // an unused split contributes weight e^(-inf) = 0
        for (int e = tid; e < grp * PART_STRIDE; e += 256) sO[e] = e % PART_STRIDE == 0 ? -INFINITY : 0.f;
    }
    if constexpr (CL) {
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        if (tr) tr[6] = gtimer();
        // every rank's partials into this CTA (all loads in flight at once, into
        // the key area), then the cluster meets once more and the peers may exit
        const int ns = (int)gridDim.x;
        float4* all = reinterpret_cast<float4*>(sK);  // [ns][ATT_MAXG * PART_STRIDE / 4]
        constexpr int PQ = ATT_MAXG * PART_STRIDE / 4;
        for (int e = tid; e < ns * PQ; e += 256) {
            const int q = e / PQ, k = e - q * PQ;
            all[e] = reinterpret_cast<const float4*>(cl.map_shared_rank(sO, q))[k];
        }
        cl.sync();
        const float* pa = reinterpret_cast<const float*>(all);
        for (int e = tid; e < ((grp - split + ns - 1) / ns) * HD; e += 256) {
            const int i = split + (e / HD) * ns, d = e % HD;
            float M = -INFINITY;
            for (int q = 0; q < ns; q++) M = fmaxf(M, pa[(q * ATT_MAXG + i) * PART_STRIDE]);
            float L = 0.f, o = 0.f;
            for (int q = 0; q < ns; q++) {
                const float* pq = pa + (q * ATT_MAXG + i) * PART_STRIDE;
                const float w = expf(pq[0] - M);
                L += pq[1] * w;
                o += pq[2 + d] * w;
            }
            a.att[(size_t)row * a.heads * HD + (kh * grp + i) * HD + d] = f2bf(rb(o * (1.0f / L)));
        }
    }
    if (tr) tr[7] = gtimer();
}

cudaError_t launch_attn(const AttnArgs& a, int rows, cudaStream_t s) {
    static int attr_set[64] = {};  // per device: the dynamic shared memory opt-ins
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaFuncSetAttribute(attn_partial_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM);
        cudaFuncSetAttribute(attn_partial_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM_CL);
        attr_set[dev] = 1;
    }
    if (!a.tmap) return cudaErrorInvalidValue;
    const bool cl = a.att && a.nsplit_max <= 8;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit_max, a.kv_heads, rows);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = cl ? ATT_SMEM_CL : ATT_SMEM;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = (unsigned)a.nsplit_max;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = cl && a.nsplit_max > 1 ? 2 : 1;
    // a cluster launch can fail where a plain one would not (e.g. the cluster's
    // shared memory does not fit); the caller checks the result
    if (cl) return cudaLaunchKernelEx(&cfg, attn_partial_kernel<true>, a, *a.tmap);
    return cudaLaunchKernelEx(&cfg, attn_partial_kernel<false>, a, *a.tmap);
}

bool attn_fused_combine(const AttnArgs& a) { return a.att && a.nsplit_max <= 8; }

// Combines the splits of each (row, head) once into att [rows][heads * 64]
// bf16, the o_proj input: o = rb(sum_s acc_s e^(m_s - M) * (1 / L)) with
// L = sum_s l_s e^(m_s - M). One CTA per (head, row), a thread per dim (each
// computes M and L itself: the split loads are the same addresses for all).
__global__ void __launch_bounds__(64) attn_combine_kernel(const float* part, RowsDev rows, int nsplit_max, int heads,
                                                          uint16_t* att) {
    const int h = blockIdx.x, row = blockIdx.y, d = threadIdx.x;
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    const int ns = (rows.pos[row] + 1 + ATT_SPLIT - 1) / ATT_SPLIT;
    const float* pr = part + ((size_t)row * nsplit_max * heads + h) * PART_STRIDE;
    const size_t ss = (size_t)heads * PART_STRIDE;  // split stride
    float M = -INFINITY;
    for (int s = 0; s < ns; s++) M = fmaxf(M, pr[s * ss]);
    float L = 0.f, o = 0.f;
#pragma unroll 4
    for (int s = 0; s < ns; s++) {
        const float* p = pr + s * ss;
        const float w = expf(p[0] - M);
        L += p[1] * w;
        o += p[2 + d] * w;
    }
    att[(size_t)row * heads * HD + h * HD + d] = f2bf(rb(o * (1.0f / L)));
}

cudaError_t launch_attn_combine(const float* part, RowsDev rows, int nsplit_max, int heads, uint16_t* att, int nrows,
                                cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(heads, nrows);
    cfg.blockDim = dim3(HD);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_combine_kernel, part, rows, nsplit_max, heads, att);
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
