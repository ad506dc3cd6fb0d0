// mega.cu — persistent decode-step kernel (see mega.cuh for the design).
#include <cuda_runtime.h>

#include "mega.cuh"

namespace ming {

namespace {

constexpr long long MG_TIMEOUT = 4000000000LL;  // cycles (~2 s) before a wait gives up
constexpr int MG_SK = MG_MAX_STAGE;             // staged 64-groups of activations (max)

// ---------------- PTX helpers ----------------
MING_DEV uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
MING_DEV void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(su32(b)), "r"(count));
}
MING_DEV void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(su32(b)), "r"(bytes) : "memory");
}
MING_DEV void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(su32(b)) : "memory");
}
MING_DEV void mbar_arrive_n(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;\n" ::"r"(su32(b)), "r"(n) : "memory");
}
MING_DEV bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
MING_DEV bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on an mbarrier phase; false on timeout. A completed phase is
// seen by the non-blocking test first.
MING_DEV bool mbar_wait(uint64_t* b, uint32_t parity) {
    if (mbar_test(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(b, parity))
        if (clock64() - t0 > MG_TIMEOUT) return false;
    return true;
}
// The producer's wait for a released slot: it runs a layer or more ahead, so
// it backs off between tests instead of competing with the consumer warps
// for issue slots and the shared-memory pipe.
MING_DEV bool mbar_wait_idle(uint64_t* b, uint32_t parity) {
    if (mbar_test(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_test(b, parity)) {
        __nanosleep(128);
        if (clock64() - t0 > MG_TIMEOUT) return false;
    }
    return true;
}
MING_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}
MING_DEV void cbar() { asm volatile("bar.sync 1, %0;\n" ::"n"(MG_CT) : "memory"); }  // consumer warps only
// Consumer barrier that also ORs one flag over the consumer threads: every
// thread gets the same answer even if the producer warp sets the flag meanwhile
MING_DEV bool cbar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(MG_CT)
        : "memory");
    return r != 0;
}
MING_DEV uint64_t ldr64(const void* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}
MING_DEV uint32_t ldr32(const void* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
MING_DEV uint4 ldcg16(const void* p) {  // 16 bytes from L2 (never a stale L1 line)
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
MING_DEV void str64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
MING_DEV void red_add64(unsigned long long* p, long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
MING_DEV uint64_t tagged(uint32_t tag, float v) { return ((uint64_t)tag << 32) | __float_as_uint(v); }
// A counted accumulator word is (contributors << 56) + sum of fixed-point
// values (|sum| < 2^55): the count (up to 255) is the top byte after
// rounding; the unsigned shift keeps counts above 127.
MING_DEV int acc_count(unsigned long long v) { return (int)((v + (1ull << 55)) >> 56); }
MING_DEV float acc_value(unsigned long long v) {
    const long long x = (long long)v - ((long long)acc_count(v) << 56);
    return __ll2float_rn(x) * (1.0f / (float)(1ull << MG_FIX));
}
// fixed point with MG_FIX fraction bits (|v| < 2^23), plus one contributor count
MING_DEV long long to_fix_counted(float v) { return __float2ll_rn(v * (float)(1ull << MG_FIX)) + (1ll << 56); }

// x / B for the step's row count B <= 4 (bm = ceil(2^32 / B)), exact for x < 2^30
MING_DEV int divB(int x, unsigned long long bm) { return (int)(((unsigned long long)(uint32_t)x * bm) >> 32); }

struct Ctx {
    const MegaDev* a;
    int* fail;  // shared: first failure code of this CTA (0 = none)
};

// Polls one tagged f32 word until its tag is `tag`. On timeout or a failure
// elsewhere, records it and returns 0 (the caller checks *fail at the next
// barrier). Kept out of line: it is the rare path of every gather.
// (Out of line and with scalar arguments: nothing of the caller's state has
// to live in local memory, which the nearly full L1 would serve from L2.)
__device__ __noinline__ float poll_word(const uint64_t* p, uint32_t tag, int* fail, const int* err) {
    uint64_t v = ldr64(p);
    if ((uint32_t)(v >> 32) == tag) return __uint_as_float((uint32_t)v);
    const long long t0 = clock64();
    int it = 0;
    while (true) {
        v = ldr64(p);
        if ((uint32_t)(v >> 32) == tag) return __uint_as_float((uint32_t)v);
        if (((++it) & 63) == 0) {
            if (*(volatile int*)fail) return 0.f;
            if (ldr32(err)) {
                atomicCAS(fail, 0, 5);
                return 0.f;
            }
            if (clock64() - t0 > MG_TIMEOUT) {
                atomicCAS(fail, 0, 1);
                return 0.f;
            }
        }
    }
}
MING_DEV float poll(const Ctx& x, const uint64_t* p, uint32_t tag) { return poll_word(p, tag, x.fail, x.a->err); }
// Four consecutive tagged words whose bf16 payloads go to dst[0], dst[B],
// dst[2B], dst[3B], each polled until it carries `tag` (the rare path of the
// SwiGLU-output gather, out of line).
__device__ __noinline__ void poll4_bf16(const uint64_t* src, uint16_t* dst, int B, uint32_t tag, int* fail, const int* err) {
    for (int u = 0; u < 4; u++) dst[u * B] = (uint16_t)__float_as_uint(poll_word(src + u, tag, fail, err));
}

// Re-reads a counted accumulator word until `expect` CTAs have contributed
// (bounded); returns the word (complete, or whatever it holds on failure).
__device__ __noinline__ unsigned long long poll_acc(const unsigned long long* p, int expect, int* fail, const int* err) {
    const long long t0 = clock64();
    int it = 0;
    while (true) {
        const unsigned long long v = ldr64(p);
        if (acc_count(v) == expect) return v;
        if (((++it) & 31) == 0) {
            if (*(volatile int*)fail) return v;
            if (ldr32(err)) {
                atomicCAS(fail, 0, 5);
                return v;
            }
            if (clock64() - t0 > MG_TIMEOUT) {
                atomicCAS(fail, 0, 1);
                return v;
            }
        }
    }
}
MING_DEV float acc_get(const Ctx& x, const unsigned long long* p, unsigned long long v, int expect) {
    if (acc_count(v) != expect) v = poll_acc(p, expect, x.fail, x.a->err);
    return acc_value(v);
}
// One thread waits for one representative word of a hand-off (so thousands
// of threads do not poll L2 while the writers work), then the CTA meets.
MING_DEV void hint_acc(const Ctx& cx, const unsigned long long* p, int expect) {
    if (threadIdx.x == 0) {
        const unsigned long long v = ldr64(p);
        if (acc_count(v) != expect) poll_acc(p, expect, cx.fail, cx.a->err);
    }
    cbar();
}

// ---------------- tensor-core groups on shared-memory chunks ----------------
// Weights of one 64-group (this lane's words + the group scales).
struct GroupW {
    uint32_t w[8];
    float s_lo, b_lo, s_hi, b_hi;
};
template <int FMT>
MING_DEV void load_group(const uint8_t* chunk, int lane, GroupW& g) {
    if constexpr (FMT == 16) {
        // bf16 tiles: 4 k-steps x this lane's uint4, loaded at use
    } else if constexpr (FMT == 4) {
        const uint4 w = *reinterpret_cast<const uint4*>(chunk + (size_t)lane * 16);
        g.w[0] = w.x; g.w[1] = w.y; g.w[2] = w.z; g.w[3] = w.w;
    } else {
        const uint4 w0 = *reinterpret_cast<const uint4*>(chunk + (size_t)lane * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(chunk + (size_t)(32 + lane) * 16);
        g.w[0] = w0.x; g.w[1] = w0.y; g.w[2] = w0.z; g.w[3] = w0.w;
        g.w[4] = w1.x; g.w[5] = w1.y; g.w[6] = w1.z; g.w[7] = w1.w;
    }
    if constexpr (FMT != 16) {
        const uint2 sc = *reinterpret_cast<const uint2*>(chunk + (FMT == 4 ? 512 : 1024) + (lane >> 2) * 8);
        g.s_lo = __uint_as_float(sc.x << 16);
        g.b_lo = __uint_as_float(sc.x & 0xffff0000u);
        g.s_hi = __uint_as_float(sc.y << 16);
        g.b_hi = __uint_as_float(sc.y & 0xffff0000u);
    }
}
template <int FMT>
MING_DEV void a_frag(const uint8_t* chunk, const GroupW& g, int ks, int lane, uint32_t (&a)[4]) {
    if constexpr (FMT == 16) {
        const uint4 w = *reinterpret_cast<const uint4*>(chunk + ((size_t)ks * 32 + lane) * 16);
        a[0] = w.x; a[1] = w.y; a[2] = w.z; a[3] = w.w;
    } else if constexpr (FMT == 4) {
        dq4(g.w[ks], a);
    } else {
        dq8(g.w[(ks >> 1) * 4 + (ks & 1) * 2], g.w[(ks >> 1) * 4 + (ks & 1) * 2 + 1], a);
    }
}
template <int FMT>
MING_DEV void mma_k(float (&t)[4], const uint32_t (&a)[4], uint2 b) {
    if constexpr (FMT == 16) mma_bf16(t, a, b.x, b.y);
    else mma_f16(t, a, b.x, b.y);
}
// acc[tu] += W_group . y_group (t: the group's own sums; the quantized scale
// and bias apply per group: s * sum(q y) + b * sum(y)). Branch-free: the
// contribution is added to both accumulators with weights 1 and 0 (exact),
// so one copy of the code serves either tile.
template <int FMT>
MING_DEV void group_finish(const GroupW& g, const float (&t)[4], const float* ys, int lane, int tu, float (&acc)[2][4]) {
    float c[4];
    if constexpr (FMT == 16) {
        c[0] = t[0]; c[1] = t[1]; c[2] = t[2]; c[3] = t[3];
    } else {
        const int cc = 2 * (lane & 3);
        const float y0 = ys[cc], y1 = ys[cc + 1];
        c[0] = g.s_lo * t[0] + g.b_lo * y0;
        c[1] = g.s_lo * t[1] + g.b_lo * y1;
        c[2] = g.s_hi * t[2] + g.b_hi * y0;
        c[3] = g.s_hi * t[3] + g.b_hi * y1;
    }
    const float m1 = tu ? 1.f : 0.f, m0 = 1.f - m1;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        acc[0][k] = fmaf(c[k], m0, acc[0][k]);
        acc[1][k] = fmaf(c[k], m1, acc[1][k]);
    }
}

// ---------------- shared memory ----------------
constexpr int MG_T_BYTES = MG_SK * 64 * MG_MAXB * 2;  // bf16 [stage][64][row]
constexpr int MG_BT_INTS = 512;                       // block-table row per batch row
constexpr int MG_B_BYTES = MG_SK * 4 * 32 * 8;        // mma B fragments
struct SmemMap {
    int ring, bars, sB, sYs, sT, sRed, sX, lp, bt, misc, total;
};
__host__ __device__ inline SmemMap smem_map(int nslots, int slot_bytes, int H, int lp_bytes) {
    SmemMap m;
    m.ring = 0;
    m.bars = nslots * slot_bytes;
    m.sB = (m.bars + (2 * nslots + 4) * 8 + 127) / 128 * 128;
    m.sYs = m.sB + MG_B_BYTES;
    m.sT = m.sYs + MG_SK * 8 * 4;
    m.sRed = m.sT + MG_T_BYTES;
    m.sX = m.sRed + MG_CWARPS * 2 * 16 * 8 * 4;
    m.lp = m.sX + (MG_MAXB * H * 2 + 127) / 128 * 128;
    m.bt = m.lp + 2 * ((lp_bytes + 127) / 128 * 128);
    m.misc = m.bt + MG_MAXB * MG_BT_INTS * 4;
    m.total = m.misc + 4096;
    return m;
}
constexpr int MG_ATT_SCRATCH = MG_B_BYTES + MG_SK * 8 * 4 + MG_T_BYTES;
// attention item scratch: K, V rows (padded to 72) + q + new k/v + scores + P.V partials
static_assert(2 * MG_ATT_CH * HD * 2 + 3 * HD * 4 + MG_ATT_CH * 4 + MG_CWARPS * 32 * 8 <= MG_ATT_SCRATCH,
              "attention scratch does not fit");
static_assert(MG_ATT_CH * HD * 2 * 2 <= MG_B_BYTES, "the attention K/V pages fit the fragment area");
static_assert(MG_ATT_CH * 4 + MG_CWARPS * 32 * 8 >= MG_CWARPS * 68 * 4, "the warps' attention partials fit the score area");

constexpr int MG_SLOT_META = 32;  // ring slots of one phase with precomputed users
struct Misc {              // small per-CTA state in shared memory
    uint64_t att_bar;            // mbarrier of the attention items' K/V page copies (first: 8-byte aligned)
    unsigned int att_uses;       // phases of att_bar completed so far
    int att_inflight;            // copies issued whose completion nobody has seen (wind-down waits for them)
    float inv[MG_MAXB];    // 1/rms of each row (current norm)
    float scl[MG_MAXB];    // operand pre-scale (power of two) of each row
    float post[MG_MAXB];   // scale applied to the f32 sums
    int pos[MG_MAXB];      // row positions (cache length before this step)
    int seq[MG_MAXB];      // row sequences
    float red[MG_CWARPS * 2 * MG_MAXB];  // block reductions
    int g0[MG_NPH], g1[MG_NPH];          // this CTA's group range per phase
    int wtile[MG_NPH][MG_CWARPS];        // first tile of each warp's group range (-1: none)
    int nsc[MG_NPH];                     // ring slots of each phase
    int pbase[MG_NPH];                   // first group's position in its tile (g0 % groups per tile)
    int grp;                             // query heads per kv head
    unsigned long long hm;               // divB multiplier of the head count
    int nitems[MG_MAXB];                 // attention items of each row: heads x 128-position chunks
    uint8_t hgrp[64];                    // kv head of each query head
    // each warp's run per phase, fixed for the whole step (computed once: the
    // integer divisions by runtime sizes cost ~0.1 us each at this kernel's
    // issue rate): groups [i0, i1) of the CTA's range, its first group's tile,
    // group in the tile and group in its ring slot, and its first and last slot
    struct WRun {
        short i0, i1, t, kg, wi, js, je, tl;  // tl: the run's last tile
    } wrun[MG_NPH][MG_CWARPS];
    float rc[MG_MAXB][HD / 2];           // RoPE cos/sin of each row's position, per frequency
    float rs[MG_MAXB][HD / 2];
    int fail;
    float om, ol;  // max and sum of this CTA's attention chunk (the combining chunk keeps its own)
    int prod_done;
    int issued;
    int frag_dirty;  // attention items reused the fragment area: rows >= B must be zeroed again
    uint32_t epoch;
    int step;
    unsigned long long bm;  // divB multiplier of the step's row count
    long long pg_el;        // elements between consecutive pages of the KV pool
    uint8_t tcount[3][MG_MAX_TILES];  // contributors per tile of the split-K phases q 0, 1, 3
    // per phase and ring slot of the phase (phases of at most MG_SLOT_META
    // slots): the lowest warp whose run uses the slot, and the arrivals it adds
    // on the slot's empty barrier for the warps that do not use it
    uint8_t sl_first[MG_NPH][MG_SLOT_META];
    uint8_t sl_extra[MG_NPH][MG_SLOT_META];
};
static_assert(sizeof(Misc) <= 4096, "Misc must fit its shared-memory slot");

struct Sm {  // shared-memory views used by the phases
    uint2* sB;
    float* sYs;
    uint16_t* sT;
    float* sRed;
    uint16_t* sX;
    const uint8_t* lp;  // current layer's parameter block
    const int* bt;      // [MG_MAXB][MG_BT_INTS]
    Misc* ms;
    long long* st;      // optional stamp row of the current layer (diagnostics)
    int so;             // stamp slot of the current phase's sub-steps
};
// Trace stamps compile only into the tracing instantiation (TR): the kernel's
// speed depends on its instruction footprint, so production code carries none.
#define MG_SUB(k) \
    if (TR && sm.st && threadIdx.x == 0) sm.st[sm.so + (k)] = clock64();

// accumulator rows of (step parity, layer, kind); row b at + b * acc_w
MING_DEV unsigned long long* acc_ptr(const MegaDev& a, uint32_t epoch, int l, int which) {
    return a.acc + (((size_t)(epoch & 1) * a.layers + l) * MG_NACC + which) * MG_MAXB * a.acc_w;
}

// ---------------- staging of the mma B operand ----------------
// Fragment entry (stage si, kstep ks, lane) holds rows b = lane/4 at
// k = si*64 + 16ks + 2t, +1, +8, +9 (t = lane%4). Entries of rows >= B are
// zero. The 16 entries of one (stage, row) are computed by 16 consecutive
// threads, which also reduce the row's group sum (the quantized formats'
// bias term) with shuffles. Sources: mode 0, sX times the norm weight nw and
// the row pre-scale; mode 1, the bf16 values sT [stage][64][row].
template <bool F16, bool TR>
MING_DEV void stage(const Sm& sm, int nstage, int B, int H, int mode, const uint16_t* nw) {
    const int tid = threadIdx.x;
    // entries of rows >= B stay zero from one stage to the next; only the
    // attention items (which reuse this area) dirty them. They are disjoint
    // from the entries written below, so no barrier separates the passes.
    if (sm.ms->frag_dirty) {
        for (int e = tid; e < MG_SK * 4 * 32; e += MG_CT)
            if ((e & 31) >= 4 * B) sm.sB[e] = make_uint2(0u, 0u);
    }
    const int tot = nstage * B * 16;
    const int totr = (tot + 31) & ~31;  // warp-uniform trip count: every lane reaches the shuffles
    for (int e = tid; e < totr; e += MG_CT) {
        const bool act = e < tot;
        const int q16 = e & 15, sb = e >> 4, si = act ? divB(sb, sm.ms->bm) : 0, b = act ? sb - si * B : 0;
        const int ks = q16 >> 2, tq = q16 & 3, kk = ks * 16 + 2 * tq;
        float sum = 0.f;
        if (act) {
            const int ko[4] = {kk, kk + 1, kk + 8, kk + 9};
            float y[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                if (mode == 0) {
                    const int f = si * 64 + ko[u];
                    y[u] = bf2f(sm.sX[b * H + f]) * bf2f(nw[f]) * sm.ms->scl[b];
                } else {
                    y[u] = bf2f(sm.sT[(si * 64 + ko[u]) * B + b]);
                }
            }
            const uint2 v = make_bfrag<F16>(y[0], y[1], y[2], y[3]);
            sm.sB[(si * 4 + ks) * 32 + b * 4 + tq] = v;
            float2 p, q;
            if (F16) {
                p = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
                q = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
            } else {
                p = unpack_bf16x2(v.x);
                q = unpack_bf16x2(v.y);
            }
            sum = (p.x + p.y) + (q.x + q.y);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if (act && q16 == 0) sm.sYs[si * 8 + b] = sum;
    }
    cbar();
    if (threadIdx.x == 0) sm.ms->frag_dirty = 0;  // read by every thread before the barrier above
    MG_SUB(0)
}

// Residual update from a fixed-point accumulator, fused with the RMSNorm
// statistics of the updated rows: sX[b][f] = rb(sX + rb(acc[b][f])), then
// inv, pre-scale and post-scale of each row for the norm weight nw. With acc
// null the rows stay as they are (the layer-0 input). Returns whether the
// CTA has failed (one answer for every consumer thread).
MING_DEV bool residual_stats(const Ctx& cx, const Sm& sm, const MegaDev& a, const unsigned long long* acc, const uint8_t* tcount,
                               const uint16_t* nw, bool f16) {
    const int H = a.H, B = a.B, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // row by row, two features per thread per pass (f = 2 tid, + 2 x 256, ...);
    // each pass's accumulator pair is requested one pass ahead, so the passes'
    // L2 round trips overlap. Kept rolled: this code runs once per layer and
    // the kernel's speed follows its instruction footprint.
#pragma unroll 1
    for (int b = 0; b < B; b++) {
        const unsigned long long* ar = acc ? acc + (size_t)b * a.acc_w : nullptr;
        uint16_t* xr = sm.sX + b * H;
        float ss = 0.f, am = 0.f;
        uint4 v = ar && tid * 2 < H ? ldcg16(ar + tid * 2) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll 1
        for (int f = tid * 2; f < H; f += 2 * MG_CT) {
            const uint4 cur = v;
            if (ar && f + 2 * MG_CT < H) v = ldcg16(ar + f + 2 * MG_CT);
            float2 x = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(xr + f));
            if (ar) {
                const int expect = tcount[f >> 4];  // f, f + 1: same tile
                const float d0 = acc_get(cx, ar + f, ((unsigned long long)cur.y << 32) | cur.x, expect);
                const float d1 = acc_get(cx, ar + f + 1, ((unsigned long long)cur.w << 32) | cur.z, expect);
                x.x = rb(x.x + rb(d0));
                x.y = rb(x.y + rb(d1));
                *reinterpret_cast<uint32_t*>(xr + f) = pack_bf16x2(x.x, x.y);
            }
            const float2 w = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(nw + f));
            ss += x.x * x.x + x.y * x.y;
            am = fmaxf(am, fmaxf(fabsf(x.x * w.x), fabsf(x.y * w.y)));
        }
        ss = warp_sum(ss);
        am = warp_max(am);
        if (lane == 0) {
            sm.ms->red[(warp * MG_MAXB + b) * 2] = ss;
            sm.ms->red[(warp * MG_MAXB + b) * 2 + 1] = am;
        }
    }
    cbar();
    if (tid < B) {
        float s1 = 0.f, a1 = 0.f;
#pragma unroll 1
        for (int w = 0; w < MG_CWARPS; w++) {
            s1 += sm.ms->red[(w * MG_MAXB + tid) * 2];
            a1 = fmaxf(a1, sm.ms->red[(w * MG_MAXB + tid) * 2 + 1]);
        }
        // e = the frexp exponent of amax / 4096 when above 1 (a normal float:
        // its biased exponent - 126), else 0; 2^-e and 2^e built from their
        // exponent bits (e stays far inside the normal range)
        int e = 0;
        if (f16 && a1 > 4096.f) e = ((__float_as_int(a1 * (1.0f / 4096.f)) >> 23) & 0xff) - 126;
        const float inv = rsqrtf(s1 / (float)H + a.eps);
        sm.ms->inv[tid] = inv;
        sm.ms->scl[tid] = __int_as_float((127 - e) << 23);
        sm.ms->post[tid] = inv * __int_as_float((127 + e) << 23);
    }
    return cbar_or(*(volatile int*)cx.fail != 0);  // the caller's failure check rides on this barrier
}

enum { OUT_ACC = 0, OUT_GLU = 1 };

// One GEMV phase on the CTA's ring chunks. Warps take contiguous runs of the
// CTA's groups (two groups per iteration: independent mma chains; a run spans
// at most two tiles), meet in shared memory, and the CTA emits per (tile,
// row, batch row) either a fixed-point contribution to acc (row index
// tile*16 + r) or, for whole gate|up tiles, the SwiGLU outputs into hb.
template <int FMT, bool TR>
MING_DEV void gemv_phase(const Ctx& cx, const Sm& sm, int p, int slot0, uint32_t par0, uint8_t* ring, uint64_t* full,
                         uint64_t* empty, int stage_base, bool use_post, int out, unsigned long long* acc, uint64_t* hb,
                         uint32_t tag) {
    const MegaDev& a = *cx.a;
    Misc* ms = sm.ms;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g0 = ms->g0[p], g1 = ms->g1[p], n = g1 - g0, gpt = a.ph[p].gpt;
    if (n <= 0) return;  // CTA-uniform
    const int nsc = ms->nsc[p];
    MG_SUB(1)
    const Misc::WRun wr = ms->wrun[p][warp];
    const int i0 = wr.i0, i1 = wr.i1;
    const int tb = ms->wtile[p][warp];
    float acc2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    // walk the warp's run incrementally: tile t, group kg in the tile, group
    // wi in its ring slot
    int t = wr.t, kg = wr.kg, wi = wr.wi;
    // The phase's ring slots one at a time: a warp waits for a slot's fill,
    // uses the groups of its run inside it and releases it (one arrival on the
    // slot's empty barrier, which expects MG_CWARPS), so a phase may be longer
    // than the ring (the producer refills released slots meanwhile).
    // With the phase inside the ring (skip mode: every use a distinct slot)
    // a warp visits only the slots of its own run. The lowest warp using a
    // slot also arrives for the warps that do not use it (sl_extra), after it
    // waited for the fill: the barrier's previous phase has completed by then
    // (the producer waited for it before refilling), and this phase completes
    // only once every user has arrived, so the producer never refills a slot
    // that is still read. Walking the other warps' slots to release them
    // cost ~0.2 us per slot per warp.
    // Otherwise every warp walks every slot in order: it releases use u+1 of
    // a slot only after waiting for its fill, which needs every warp's
    // release of use u, so arrivals of two uses never mix.
    const bool skip = nsc <= a.nslots && nsc <= MG_SLOT_META;
    const int js = i0 < i1 ? wr.js : 0, je = i0 < i1 ? wr.je : -1;
    const int njj = skip ? je - js + 1 : nsc;
    // slot of phase slot jj: slot0 + jj, wrapped once at most in skip mode;
    // in order (one wrap per pass of the ring) otherwise
    int sl = slot0;
    uint32_t par = par0;
#pragma unroll 1
    for (int it = 0; it < njj; it++) {
        int jj = it;
        if (skip) {
            jj = js + it;
            sl = slot0 + jj;
            par = par0;
            if (sl >= a.nslots) {
                sl -= a.nslots;
                par ^= 1u;
            }
        } else if (it > 0 && ++sl == a.nslots) {
            sl = 0;
            par ^= 1u;
        }
        const int w0 = max(i0, jj * a.gps), w1 = min(i1, (jj + 1) * a.gps);
        if ((!skip || w0 < w1) && !mbar_wait(&full[sl], par)) atomicCAS(cx.fail, 0, 2);
        if (TR && sm.st && (MG_CWARPS <= 8 || warp < 8) && lane == 0 && p == 2 && w0 == i0 && w0 < w1) sm.st[56 + warp] = clock64();
        if (w0 < w1 && !*(volatile int*)cx.fail) {
            const uint8_t* sbase = ring + (size_t)sl * a.slot_bytes;
#pragma unroll 1
            for (int i = w0; i < w1; i += 2) {
                const bool two = i + 1 < w1;
                const uint8_t* ch[2];
                int si[2], tu[2];
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    if (u == 1 && !two) {
                        ch[1] = ch[0];
                        si[1] = si[0];
                        tu[1] = tu[0];
                        break;
                    }
                    ch[u] = sbase + (size_t)wi * a.cb;
                    const int s_ = kg - stage_base;
                    si[u] = s_ < 0 ? s_ + gpt : s_;
                    tu[u] = t == tb ? 0 : 1;
                    if (++kg == gpt) {
                        kg = 0;
                        t++;
                    }
                    if (++wi == a.gps) wi = 0;
                }
                GroupW gw[2];
                load_group<FMT>(ch[0], lane, gw[0]);
                load_group<FMT>(ch[1], lane, gw[1]);
                float t0[4] = {0.f, 0.f, 0.f, 0.f}, t1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int ks = 0; ks < 4; ks++) {
                    uint32_t a0[4], a1[4];
                    a_frag<FMT>(ch[0], gw[0], ks, lane, a0);
                    a_frag<FMT>(ch[1], gw[1], ks, lane, a1);
                    const uint2 b0 = sm.sB[(si[0] * 4 + ks) * 32 + lane];
                    const uint2 b1 = sm.sB[(si[1] * 4 + ks) * 32 + lane];
                    mma_k<FMT>(t0, a0, b0);
                    mma_k<FMT>(t1, a1, b1);
                }
                group_finish<FMT>(gw[0], t0, sm.sYs + si[0] * 8, lane, tu[0], acc2);
                if (two) group_finish<FMT>(gw[1], t1, sm.sYs + si[1] * 8, lane, tu[1], acc2);
            }
        }
        __syncwarp();
        if (lane == 0) {  // before any global write of this phase
            if (skip && ms->sl_first[p][jj] == warp) mbar_arrive_n(&empty[sl], 1u + ms->sl_extra[p][jj]);
            else mbar_arrive(&empty[sl]);
        }
        if (TR && sm.st && (MG_CWARPS <= 8 || warp < 8) && lane == 0 && p >= 2 && w1 == i1 && w0 < w1) sm.st[40 + (p - 2) * 8 + warp] = clock64();
    }
    MG_SUB(2)
    const int B = a.B;
    if (out == OUT_ACC) {
        // split-K phases: each warp adds its own partial sums of the (at most
        // two) tiles its run touched; the tiles' contributor counts count
        // warps (planned on the host), so no CTA-wide reduction is needed
        if (i0 < i1) {
            const int gr = lane >> 2, cc = 2 * (lane & 3), tl = wr.tl;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int t = tb + u;
                if (u == 1 && t > tl) break;
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int b = cc + j;
                    if (b >= B) continue;
                    const float ps = use_post ? ms->post[b] : 1.f;
                    unsigned long long* base = acc + (size_t)b * a.acc_w + t * 16;
                    red_add64(base + gr, to_fix_counted(acc2[u][j] * ps));
                    red_add64(base + gr + 8, to_fix_counted(acc2[u][2 + j] * ps));
                }
            }
        }
        if (TR && sm.st && (MG_CWARPS <= 8 || warp < 8) && lane == 0) sm.st[64 + (p < 3 ? p : 2) * 8 + warp] = clock64();
        MG_SUB(4)
        return;
    }
    {
        const int gr = lane >> 2, cc = 2 * (lane & 3);
        float* r = sm.sRed + warp * 2 * 128;
#pragma unroll
        for (int u = 0; u < 2; u++) {
            r[u * 128 + gr * 8 + cc] = acc2[u][0];
            r[u * 128 + gr * 8 + cc + 1] = acc2[u][1];
            r[u * 128 + (gr + 8) * 8 + cc] = acc2[u][2];
            r[u * 128 + (gr + 8) * 8 + cc + 1] = acc2[u][3];
        }
    }
    cbar();
    MG_SUB(3)
    const int t0 = g0 / gpt, nt = (g1 - 1) / gpt - t0 + 1;
    {
        // whole gate|up tiles: rows 0..7 gate, 8..15 up of features 8t..8t+7
        for (int e = threadIdx.x; e < nt * 32; e += MG_CT) {
            const int b = e & 3, r = (e >> 2) & 7, t = t0 + (e >> 5);
            if (b >= B) continue;
            float gs = 0.f, us = 0.f;
#pragma unroll
            for (int w = 0; w < MG_CWARPS; w++) {
                const int wt = ms->wtile[p][w];
                const float g0 = sm.sRed[(w * 2 + 0) * 128 + r * 8 + b], g1 = sm.sRed[(w * 2 + 1) * 128 + r * 8 + b];
                const float u0 = sm.sRed[(w * 2 + 0) * 128 + (r + 8) * 8 + b], u1 = sm.sRed[(w * 2 + 1) * 128 + (r + 8) * 8 + b];
                const bool in0 = wt == t, in1 = wt >= 0 && wt + 1 == t;
                gs += in0 ? g0 : (in1 ? g1 : 0.f);
                us += in0 ? u0 : (in1 ? u1 : 0.f);
            }
            const float gv = rb(gs * ms->post[b]), uv = rb(us * ms->post[b]);
            const float sg = rb(1.0f / (1.0f + expf(-gv)));
            str64(hb + (size_t)b * a.FF + t * 8 + r, ((uint64_t)tag << 32) | f2bf(rb(rb(gv * sg) * uv)));
        }
    }
    MG_SUB(4)
}

// The combine's per-dim partial sums of the MG_NQ thread groups, in a fixed
// order (pairwise for four groups).
MING_DEV float sum_groups(const float* red, int d) {
    if constexpr (MG_NQ == 4) {
        return (red[d] + red[64 + d]) + (red[128 + d] + red[192 + d]);
    } else {
        float o = red[d];
#pragma unroll
        for (int q = 1; q < MG_NQ; q++) o += red[q * 64 + d];
        return o;
    }
}

// Attention of one (row, query head, 128-position chunk) item. q of the head
// and the kv group's new k, v come from the q|k|v accumulator (+ bias, bf16,
// RoPE on q and k as MLX fast_rope); the chunk's cached K/V rows are
// prefetched with cp.async before the wait for q|k|v. The first head of the
// group appends the new position to the cache (in the chunk holding it).
template <bool TR>
MING_DEV void attention_item(const Ctx& cx, const Sm& sm, int l, uint32_t tag, int b, int h, int s, bool waited) {
    const MegaDev& a = *cx.a;
    Misc* ms = sm.ms;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = ms->grp, g = ms->hgrp[h], pos = ms->pos[b];
    const int p0 = s * MG_ATT_CH, p1 = min(pos + 1, p0 + MG_ATT_CH), pc = min(p1, pos), len = p1 - p0;
    const int ns = (pos + MG_ATT_CH) / MG_ATT_CH;  // chunks of the (row, head); chunk ns - 1 combines them
    // K/V rows as the pool stores them (16-position pages of [16][64] bf16,
    // 128 B per row), one bulk copy per page
    constexpr int KS = HD;
    uint16_t* sK = reinterpret_cast<uint16_t*>(sm.sB);         // [128][64]
    uint16_t* sV = sK + MG_ATT_CH * KS;                          // [128][64]
    float* sq = reinterpret_cast<float*>(sV + MG_ATT_CH * KS);  // [64] q, pre-scaled by 1/8
    float* sS = sq + HD;                                         // scores, warp partials, the combine
    const int* bt = sm.bt + b * MG_BT_INTS;
    if (tid == 0) ms->frag_dirty = 1;
    // 1. prefetch the pages holding cached positions [p0, pc): one 2 KB bulk
    //    copy per page and K/V (p0 is page-aligned; rows of a partial last
    //    page past pc are never read), completing on the CTA's attention
    //    mbarrier. Every thread read the barrier's phase count before the
    //    barrier that follows (thread 0 advances it there).
    const uint32_t att_par = ms->att_uses & 1u;
    if (TR && sm.st && tid == 0) sm.st[90] = clock64();  // diagnostics: item start (page copies issued next)
    if (tid == 0) {
        const int npg = (pc - p0 + PAGE - 1) / PAGE;
        constexpr uint32_t PG = PAGE * HD * 2;
        // earlier generic-proxy accesses of this area (fragments, the last
        // item's rows) are ordered before the copies' async-proxy writes
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        if (npg > 0) {
            mbar_expect_tx(&ms->att_bar, (uint32_t)npg * 2u * PG);
            // the (layer, K, kv head) block of page 0; pages ms->pg_el
            // elements apart, V kv_heads x 1024 elements after K
            const uint16_t* k0 = a.kv.pool + ((l * 2) * a.kvh + g) * (PAGE * HD);
            const uint32_t bar = su32(&ms->att_bar), d0 = su32(sK);
#pragma unroll 1
            for (int i = 0; i < npg; i++) {
                const uint16_t* kp = k0 + (size_t)bt[(p0 >> 4) + i] * ms->pg_el;
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%4], [%5], %2, [%3];\n" ::"r"(d0 + i * PG),
                    "l"(kp), "r"(PG), "r"(bar), "r"(d0 + MG_ATT_CH * HD * 2 + i * PG), "l"(kp + a.kvh * (PAGE * HD))
                    : "memory");
            }
        } else {
            mbar_arrive(&ms->att_bar);  // nothing cached in this chunk: complete the phase
        }
        ms->att_inflight = 1;
    }
    // 2. q of the head, k, v of the new position: entry (kind, tile, r8) holds
    //    the RoPE pair (d, d+32) = tile rows r8, r8 + 8
    const unsigned long long* qacc = acc_ptr(a, ms->epoch, l, MG_ACC_QKV) + (size_t)b * a.acc_w;
    if (!waited) hint_acc(cx, qacc + (size_t)(a.ph[0].tiles - 1) * 16 + 15, ms->tcount[0][a.ph[0].tiles - 1]);
    const float* bias = reinterpret_cast<const float*>(sm.lp + 4 * a.H);
    const int kind = tid >> 5, dq = ((tid >> 3) & 3) * 8 + (tid & 7);  // this thread's q|k|v dims dq, dq + 32
    uint16_t kv1 = 0, kv2 = 0;  // kind 1 / 2: the new key / value pair (dims d, d + 32) in bf16
    if (tid < 96) {
        const int tl = (tid >> 3) & 3, r8 = tid & 7;
        const int t = kind == 0 ? h * 4 + tl : (kind == 1 ? a.heads * 4 + g * 4 + tl : a.heads * 4 + a.kvh * 4 + g * 4 + tl);
        const uint64_t vlo = ldr64(qacc + t * 16 + r8), vhi = ldr64(qacc + t * 16 + r8 + 8);
        const int expect = ms->tcount[0][t];
        float x1 = rb(acc_get(cx, qacc + t * 16 + r8, vlo, expect) + bias[t * 16 + r8]);
        float x2 = rb(acc_get(cx, qacc + t * 16 + r8 + 8, vhi, expect) + bias[t * 16 + r8 + 8]);
        if (kind < 2) {
            const float cs = ms->rc[b][dq], sn = ms->rs[b][dq];
            const float p_ = x1 * cs - x2 * sn, q_ = x1 * sn + x2 * cs;
            x1 = rb(p_);
            x2 = rb(q_);
        }
        if (kind == 0) {
            sq[dq] = 0.125f * x1;
            sq[dq + 32] = 0.125f * x2;
        } else {
            kv1 = f2bf(x1);
            kv2 = f2bf(x2);
        }
    }
    if (TR && sm.st && tid == 0) sm.st[88] = clock64();  // diagnostics: q, k, v in registers
    if (!mbar_wait(&ms->att_bar, att_par)) atomicCAS(cx.fail, 0, 6);
    if (TR && sm.st && tid == 0) sm.st[89] = clock64();  // diagnostics: K/V pages landed
    // 3. in the chunk holding the new position, its key and value go into
    //    their rows of sK / sV (after this thread saw the page copies land:
    //    the rows are then read like every cached one), and the group's first
    //    head appends them to the cache
    if (kind >= 1 && kind <= 2 && p1 == pos + 1) {
        uint16_t* row = (kind == 1 ? sK : sV) + (pos - p0) * KS;
        row[dq] = kv1;
        row[dq + 32] = kv2;
        if (h % grp == 0) {
            uint16_t* dst = a.kv.pool + kv_index(a.kv, bt[pos / PAGE], l, kind - 1, g, pos % PAGE);
            dst[dq] = kv1;
            dst[dq + 32] = kv2;
        }
    }
    cbar();
    if (tid == 0) {
        ms->att_uses++;
        if (!*(volatile int*)cx.fail) ms->att_inflight = 0;
    }
    if (TR && sm.st && tid == 0) sm.st[36] = clock64();  // diagnostics: q, k, v and the chunk's K/V in shared memory
    // 4. each warp takes 16 positions of the chunk, 16 w.. 16 w + 15, and runs
    //    scores, softmax and P.V on them with no CTA barrier between the
    //    steps: lane (j = lane & 15, half = lane >> 4) dots half of the head
    //    dims of position 16 w + j, the halves meet by one shuffle
    static_assert(MG_ATT_CH == 16 * MG_CWARPS, "attention: 16 positions per consumer warp");
    const int jw = warp * 16 + (lane & 15), half = lane >> 4;
    float sc = -INFINITY;
    if (jw < len) {
        // rows are 128 B apart: lane (j, half) reads its 16-byte pieces in
        // the order c = (q + j) & 3, so each read instruction spreads the
        // warp over all eight bank groups
        float s0 = 0.f, s1 = 0.f;
        const float* qh = sq + 32 * half;
        const uint4* src = reinterpret_cast<const uint4*>(sK + jw * KS + 32 * half);
#pragma unroll
        for (int q0 = 0; q0 < 4; q0++) {
            const int q = (q0 + jw) & 3;
            const uint4 v = src[q];
            const float4 qa = *reinterpret_cast<const float4*>(qh + 8 * q);
            const float4 qb = *reinterpret_cast<const float4*>(qh + 8 * q + 4);
            const float2 k0 = unpack_bf16x2(v.x), k1 = unpack_bf16x2(v.y), k2 = unpack_bf16x2(v.z), k3 = unpack_bf16x2(v.w);
            s0 += qa.x * k0.x + qa.y * k0.y + qa.z * k1.x + qa.w * k1.y;
            s1 += qb.x * k2.x + qb.y * k2.y + qb.z * k3.x + qb.w * k3.y;
        }
        sc = s0 + s1;
    }
    sc += __shfl_xor_sync(0xffffffffu, sc, 16);  // both halves hold the position's score
    float m = sc;
#pragma unroll
    for (int o = 8; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (TR && sm.st && tid == 0) sm.st[15] = clock64();  // diagnostics: warp 0's scores and maximum
    const float pj = jw < len ? expf(sc - m) : 0.f;  // m is finite wherever some position is valid
    float lsum = pj;
#pragma unroll
    for (int o = 8; o; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    // P.V: lane = dim pair (2 lane, 2 lane + 1) over the warp's valid
    // positions; the probabilities go through the warp's slot of the partial
    // area (floats 4..19, overwritten only after the __syncwarp below) and
    // are read four at a time
    const int nj = max(0, min(16, len - warp * 16));  // warp-uniform
    float* ps = sS + warp * 68 + 4;
    if (lane < 16) ps[lane] = pj;
    __syncwarp();
    float2 ac = make_float2(0.f, 0.f);
#pragma unroll 1
    for (int j4 = 0; j4 < nj; j4 += 4) {
        const float4 p4 = *reinterpret_cast<const float4*>(ps + j4);
        const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int j = j4 + i;
            if (j < nj) {  // rows past the chunk's length are never read
                const float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(sV + (warp * 16 + j) * KS + 2 * lane));
                ac.x += pv[i] * v.x;
                ac.y += pv[i] * v.y;
            }
        }
    }
    __syncwarp();  // every lane read the probabilities before the partials overwrite them
    if (TR && sm.st && tid == 0) sm.st[16] = clock64();  // diagnostics: warp 0's P.V done
    // the warps' (max, sum, P.V) partials meet in shared memory (the score
    // area); 64 threads, one per dim, merge them into the chunk's partial
    float* wp = sS;  // [MG_CWARPS][68] (the probabilities above lived in floats 4..19 of each warp's row)
    if (lane == 0) {
        wp[warp * 68] = nj > 0 ? m : -INFINITY;
        wp[warp * 68 + 1] = lsum;
    }
    wp[warp * 68 + 2 + 2 * lane] = ac.x;
    wp[warp * 68 + 3 + 2 * lane] = ac.y;
    cbar();
    if (TR && sm.st && tid == 0) sm.st[37] = clock64();  // diagnostics: every warp's partial in shared memory
    float* own = sq;  // [64] this chunk's P.V sums when it combines (q is no longer read)
    if (tid < HD) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < MG_CWARPS; w++) M = fmaxf(M, wp[w * 68]);
        float L = 0.f, o = 0.f;
#pragma unroll 1
        for (int w = 0; w < MG_CWARPS; w++) {
            const float mw = wp[w * 68];
            const float e = mw == -INFINITY ? 0.f : expf(mw - M);
            L += wp[w * 68 + 1] * e;
            o += wp[w * 68 + 2 + tid] * e;
        }
        if (s == ns - 1) {
            own[tid] = o;
            if (tid == 0) {
                ms->om = M;
                ms->ol = L;
            }
        } else {
            uint64_t* ob = a.attn + (((size_t)b * a.heads + h) * a.max_splits + s) * MG_PART;
            if (tid == 0) {
                str64(ob, tagged(tag, M));
                str64(ob + 1, tagged(tag, L));
            }
            str64(ob + 2 + tid, tagged(tag, o));
        }
    }
    if (s != ns - 1) return;  // CTA-uniform; the caller meets at a barrier next
    cbar();  // own, om, ol written; the score area is free for the combine below
    // 7. the chunk holding the new position combines the (row, head):
    //    o = sum_s acc_s e^(m_s - M) / L over the other chunks' tagged partials
    //    (each word polled until this step's tag shows; every chunk with a
    //    smaller item index runs on some CTA, so the wait ends) and its own
    //    sums, then publishes the 64 values for every o_proj CTA that reads
    //    this head. Thread (d, quarter) sums the chunks s = quarter, quarter +
    //    4, ... of dim d; the values are loaded once the chunk maxima and
    //    sums have shown up (written in the same pass, so they are rarely
    //    stale; loading them earlier found them stale and polled each one)
    const int no = ns - 1;
    const uint64_t* ob = a.attn + ((size_t)b * a.heads + h) * a.max_splits * MG_PART;
    float* cm = sS;       // [no] chunk maxima (scores are no longer read)
    float* cl = sS + 64;  // [no] chunk sums
    const int d = tid & 63, qt = tid >> 6;  // qt < MG_NQ
    uint64_t va[4];
    if (tid < 2 * no) {
        const uint64_t* w = ob + (size_t)(tid >> 1) * MG_PART + (tid & 1);
        const uint64_t v = ldr64(w);
        (tid & 1 ? cl : cm)[tid >> 1] = (uint32_t)(v >> 32) == tag ? __uint_as_float((uint32_t)v) : poll(cx, w, tag);
    }
    cbar();
    if (TR && sm.st && tid == 0) sm.st[38] = clock64();  // diagnostics: the other chunks' maxima and sums in hand
    // the first pass's values are requested before the maxima and sums are
    // combined (M first, then L = sum_s l_s e^(m_s - M) in chunk order)
#pragma unroll
    for (int k = 0; k < 4; k++) va[k] = qt + MG_NQ * k < no ? ldr64(ob + (size_t)(qt + MG_NQ * k) * MG_PART + 2 + d) : 0ull;
    float M = ms->om;
    for (int q = 0; q < no; q++) M = fmaxf(M, cm[q]);
    float L = 0.f;
    for (int q = 0; q < no; q++) L += cl[q] * expf(cm[q] - M);
    L += ms->ol * expf(ms->om - M);
    const float il = 1.0f / L;
    float v = 0.f;
    // the four loads of a pass are in flight together; a stale word is
    // polled on its own
#pragma unroll 1
    for (int s0 = qt; s0 < no; s0 += 4 * MG_NQ) {
        if (s0 != qt) {
#pragma unroll
            for (int k = 0; k < 4; k++) va[k] = s0 + MG_NQ * k < no ? ldr64(ob + (size_t)(s0 + MG_NQ * k) * MG_PART + 2 + d) : 0ull;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int sk = s0 + MG_NQ * k;
            if (sk >= no) continue;
            const uint64_t* w = ob + (size_t)sk * MG_PART + 2 + d;
            const float x = (uint32_t)(va[k] >> 32) == tag ? __uint_as_float((uint32_t)va[k]) : poll(cx, w, tag);
            v += x * (expf(cm[sk] - M) * il);
        }
    }
    float* red = cl + 64;  // [4][64], in the score area (the warp partials were read before the barriers above)
    red[qt * 64 + d] = v;
    cbar();
    if (tid < HD) {
        const float o = sum_groups(red, tid) + own[tid] * (expf(ms->om - M) * il);
        str64(a.comb + ((size_t)b * a.heads + h) * HD + tid, tagged(tag, rb(o)));
    }
    if (TR && sm.st && tid == 0 && l > 0) sm.st[39] = clock64();  // diagnostics: head published (slot 39 of layer 0 is the origin)
}

// o_proj input: the combined attention output of the heads this CTA's
// o_proj range reads (published by each head's last chunk), into sT
// [si][d][b]. Returns whether the CTA has failed.
MING_DEV bool combine_heads(const Ctx& cx, const Sm& sm, int nst, int base, int gpt, uint32_t tag) {
    const MegaDev& a = *cx.a;
    Misc* ms = sm.ms;
    const int B = a.B, tot = nst * 64 * B;
    for (int e = threadIdx.x; e < tot; e += MG_CT) {
        const int qd = divB(e, ms->bm), b = e - qd * B, si = qd >> 6, d = qd & 63;
        const int h = si + base < gpt ? si + base : si + base - gpt;
        const uint64_t* p = a.comb + ((size_t)b * a.heads + h) * HD + d;
        const uint64_t v = ldr64(p);
        sm.sT[e] = f2bf((uint32_t)(v >> 32) == tag ? __uint_as_float((uint32_t)v) : poll(cx, p, tag));
    }
    return cbar_or(*(volatile int*)cx.fail != 0);
}

template <int FMT, bool TR>
__global__ void __launch_bounds__(MG_THREADS, 1) mega_kernel(const __grid_constant__ MegaDev a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const SmemMap mp = smem_map(a.nslots, a.slot_bytes, a.H, a.lp_bytes);
    uint8_t* ring = smem + mp.ring;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + mp.bars);
    uint64_t* empty = full + a.nslots;
    uint64_t* lp_full = empty + a.nslots;  // [2]
    uint64_t* lp_empty = lp_full + 2;      // [2]
    uint8_t* lpbuf = smem + mp.lp;
    const int lp_stride = (a.lp_bytes + 127) / 128 * 128;
    int* btab = reinterpret_cast<int*>(smem + mp.bt);
    Misc* ms = reinterpret_cast<Misc*>(smem + mp.misc);
    Sm sm{reinterpret_cast<uint2*>(smem + mp.sB), reinterpret_cast<float*>(smem + mp.sYs),
          reinterpret_cast<uint16_t*>(smem + mp.sT), reinterpret_cast<float*>(smem + mp.sRed),
          reinterpret_cast<uint16_t*>(smem + mp.sX), lpbuf, btab, ms, nullptr, 0};
    const int tid = threadIdx.x, c = blockIdx.x, H = a.H, B = a.B;
    constexpr bool F16 = FMT != 16;
    // ---- set-up: barriers, this CTA's ranges, block-table rows, RoPE table ----
    if (tid == 0) {
        for (int i = 0; i < a.nslots; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], MG_CWARPS);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&lp_full[i], 1);
            mbar_init(&lp_empty[i], 1);
        }
        mbar_init(&ms->att_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        ms->att_uses = 0;
        ms->att_inflight = 0;
        ms->fail = 0;
        ms->frag_dirty = 1;
        ms->prod_done = 0;
        ms->issued = 0;
        ms->epoch = (uint32_t)a.counter[0] + 1u;
        ms->step = a.counter[1];
        ms->bm = ((1ull << 32) + (unsigned long long)B - 1ull) / (unsigned long long)B;
    }
    if (tid < MG_NPH) {
        ms->g0[tid] = a.ph[tid].cta_g0[c];
        ms->g1[tid] = a.ph[tid].cta_g0[c + 1];
    }
    if (tid < B) {
        const int sq = a.row_seq[tid];
        ms->seq[tid] = sq;
        ms->pos[tid] = a.seq_len[sq];
    }
    __syncthreads();
    for (int b = 0; b < B; b++) {
        const int np = ms->pos[b] / PAGE + 1;
        for (int i = tid; i < np; i += MG_THREADS) btab[b * MG_BT_INTS + i] = a.kv.bt[(size_t)ms->seq[b] * a.kv.bt_ld + i];
    }
    if (tid < B * (HD / 2)) {
        // MLX fast_rope angles: pos * 2^(-(d/32) log2 theta), f32
        const int b = tid / (HD / 2), d = tid % (HD / 2);
        const float th = (float)ms->pos[b] * exp2f(-((float)d / 32.0f) * a.log2_theta);
        float sn, cs;
        sincosf(th, &sn, &cs);
        ms->rc[b][d] = cs;
        ms->rs[b][d] = sn;
    }
    for (int i = tid; i < 3 * MG_MAX_TILES; i += MG_THREADS) {
        const int q = i / MG_MAX_TILES, t = i % MG_MAX_TILES, p = q == 0 ? 0 : (q == 1 ? 1 : 3);
        ms->tcount[q][t] = (uint8_t)(t < a.ph[p].tiles ? a.ph[p].tcount[t] : 0);
    }
    if (tid < MG_NPH * MG_CWARPS) {
        const int p = tid / MG_CWARPS, w = tid % MG_CWARPS, n = ms->g1[p] - ms->g0[p], gpt = a.ph[p].gpt;
        const int i0 = w * n / MG_CWARPS, i1 = (w + 1) * n / MG_CWARPS;
        ms->wtile[p][w] = i1 > i0 ? (ms->g0[p] + i0) / gpt : -1;
        Misc::WRun r{};
        r.i0 = (short)i0;
        r.i1 = (short)i1;
        r.je = -1;
        if (i1 > i0) {
            const int g = ms->g0[p] + i0;
            r.t = (short)(g / gpt);
            r.kg = (short)(g - r.t * gpt);
            r.wi = (short)(i0 % a.gps);
            r.js = (short)(i0 / a.gps);
            r.je = (short)((i1 - 1) / a.gps);
            r.tl = (short)((ms->g0[p] + i1 - 1) / gpt);
        }
        ms->wrun[p][w] = r;
        if (w == 0) {
            ms->nsc[p] = n > 0 ? (n + a.gps - 1) / a.gps : 0;
            ms->pbase[p] = ms->g0[p] % gpt;
        }
    }
    if (tid < 64) ms->hgrp[tid] = (uint8_t)(tid < a.heads ? tid / (a.heads / a.kvh) : 0);
    if (tid < B) ms->nitems[tid] = a.heads * ((ms->pos[tid] + MG_ATT_CH) / MG_ATT_CH);
    if (tid == 0) {
        ms->pg_el = (long long)a.layers * 2 * a.kvh * (PAGE * HD);
        ms->grp = a.heads / a.kvh;
        ms->hm = ((1ull << 32) + (unsigned long long)a.heads - 1ull) / (unsigned long long)a.heads;
    }
    __syncthreads();
    if (tid < MG_NPH) {
        const int p = tid;
        for (int jj = 0; jj < ms->nsc[p] && jj < MG_SLOT_META; jj++) {
            int users = 0, first = 0;
            for (int w = MG_CWARPS - 1; w >= 0; w--) {
                const Misc::WRun r = ms->wrun[p][w];
                if (r.i0 < r.i1 && r.js <= jj && jj <= r.je) {
                    users++;
                    first = w;
                }
            }
            ms->sl_first[p][jj] = (uint8_t)first;
            ms->sl_extra[p][jj] = (uint8_t)(MG_CWARPS - users);
        }
    }
    __syncthreads();
    const uint32_t epoch = ms->epoch;

    // ---------------- producer warp: stream this CTA's weight ranges ----------------
    if (tid >= MG_CT) {
        if (tid == MG_CT) {
            int sc = 0;
            bool ok = true;
            for (int l = 0; l < a.layers && ok; l++) {
                const int lb = l & 1;  // the layer's parameter block, double-buffered
                if (l >= 2 && !mbar_wait_idle(&lp_empty[lb], ((l >> 1) - 1) & 1)) {
                    atomicCAS(&ms->fail, 0, 3);
                    break;
                }
                mbar_expect_tx(&lp_full[lb], (uint32_t)a.lp_bytes);
                bulk_g2s(lpbuf + lb * lp_stride, a.lparams + (size_t)l * a.lp_bytes, (uint32_t)a.lp_bytes, &lp_full[lb]);
                for (int p = 0; p < MG_NPH && ok; p++) {
                    const int g0 = ms->g0[p], n = ms->g1[p] - g0;
                    const uint8_t* src = a.wbase[l * MG_NPH + p] + (size_t)g0 * a.cb;
                    for (int j = 0; j * a.gps < n; j++, sc++) {
                        const int slot = sc % a.nslots;
                        if (sc >= a.nslots && !mbar_wait_idle(&empty[slot], ((sc / a.nslots) - 1) & 1)) {
                            atomicCAS(&ms->fail, 0, 3);
                            ok = false;
                            break;
                        }
                        if (*(volatile int*)&ms->fail) {
                            ok = false;
                            break;
                        }
                        const int ng = min(a.gps, n - j * a.gps);
                        const uint32_t bytes = (uint32_t)(ng * a.cb);
                        mbar_expect_tx(&full[slot], bytes);
                        bulk_g2s(ring + (size_t)slot * a.slot_bytes, src + (size_t)j * a.gps * a.cb, bytes, &full[slot]);
                        *(volatile int*)&ms->issued = sc + 1;
                    }
                }
            }
            *(volatile int*)&ms->prod_done = 1;
        }
        return;
    }

    // ---------------- consumer warps ----------------
    Ctx cx{&a, &ms->fail};
    int cons = 0, lp_used = 0;  // ring slots consumed so far (the wind-down waits for those issued after)
    int cslot = 0;                // cons % nslots and the parity of cons / nslots, kept without dividing
    uint32_t cpar = 0;
    bool dead = false;
    auto check = [&]() -> bool {
        if (cbar_or(*(volatile int*)&ms->fail != 0)) dead = true;  // every consumer thread sees the same answer
        return dead;
    };
    {
        // zero this CTA's slice of the accumulators of the next step (the
        // previous step used them; this step's were zeroed by it)
        const size_t per = (size_t)a.layers * MG_NACC * MG_MAXB * a.acc_w;  // int64 per parity
        uint4* z = reinterpret_cast<uint4*>(a.acc + (size_t)((epoch + 1) & 1) * per);
        const size_t n2 = per / 2, lo = n2 * c / a.C, hi = n2 * (c + 1) / a.C;
        for (size_t i = lo + tid; i < hi; i += MG_CT) z[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    for (int idx = tid; idx < B * H; idx += MG_CT) sm.sX[idx] = a.x_in[idx];
    cbar();
    long long* tr = TR && a.trace ? a.trace + (size_t)c * a.layers * MG_TRACE : nullptr;
    if (TR && tr && tid == 0) {
        // diagnostics only: a common time origin for every CTA's clock64
        // stamps. Each CTA arrives on a counter after the trace rows; the
        // clock64 at which a CTA sees all C arrivals (within an L2 round trip
        // of the others) goes to slot 39 of its layer-0 row. Bounded wait; the
        // counter holds epoch x C after every traced step.
        unsigned int* sync = reinterpret_cast<unsigned int*>(a.trace + (size_t)a.C * a.layers * MG_TRACE);
        atomicAdd(sync, 1u);
        const unsigned int target = epoch * (unsigned int)a.C;
        const long long t0 = clock64();
        while (ldr32(sync) < target && clock64() - t0 < MG_TIMEOUT) {
        }
        tr[39] = clock64();
    }
#define MG_STAMP(k) \
    if (TR && tr && tid == 0) tr[l * MG_TRACE + (k)] = clock64();
#pragma unroll 1
    for (int l = 0; l < a.layers && !dead; l++) {
        const uint32_t tag = epoch * 32u + (uint32_t)l;
        uint64_t* hb = a.hbuf + (size_t)l * MG_MAXB * a.FF;
        sm.st = tr ? tr + l * MG_TRACE : nullptr;
        MG_STAMP(0)
        if (!mbar_wait(&lp_full[l & 1], (l >> 1) & 1)) atomicCAS(cx.fail, 0, 2);
        lp_used = l + 1;
        sm.lp = lpbuf + (l & 1) * lp_stride;
        const uint16_t* ln1 = reinterpret_cast<const uint16_t*>(sm.lp);
        const uint16_t* ln2 = ln1 + H;
        // The four GEMV phases share one copy of their code (the kernel's
        // instruction footprint per layer decides its speed):
        //   q 0: x = x1(l-1) + down(l-1), RMSNorm folded, q|k|v -> acc QKV
        //   q 1: attention over the cache (P1), chunk combine, o_proj -> acc X1
        //   q 2: x1 = x + o_proj, RMSNorm folded, gate|up tiles -> SwiGLU h
        //   q 3: h of this CTA's down range, down -> acc X2
#pragma unroll 1
        for (int q = 0; q < MG_NPH && !dead; q++) {
            const int gpt = a.ph[q].gpt, n = ms->g1[q] - ms->g0[q];
            const bool rows = q == 0 || q == 2;  // input = the normed residual rows
            int base = 0, nst = H / 64;
            if (!rows) {
                base = ms->pbase[q];
                nst = min(n, gpt);
            }
            if (q == 1) {
                // P1: attention items (row, chunk, query head) strided over the
                // CTAs; neighbouring CTAs share a chunk's K/V lines in L2
                int tot = 0;
                for (int b = 0; b < B; b++) tot += ms->nitems[b];
                bool waited = false;
                for (int it = c; it < tot && !dead; it += a.C) {
                    int rem = it, b = 0;
                    while (rem >= ms->nitems[b]) {
                        rem -= ms->nitems[b];
                        b++;
                    }
                    const int sch = divB(rem, ms->hm);  // rem / heads (rem < 2^16: exact)
                    attention_item<TR>(cx, sm, l, tag, b, rem - sch * a.heads, sch, waited);
                    waited = true;
                    check();  // the next item reuses the shared-memory areas
                }
                if (dead) break;
                MG_STAMP(9)
                if (combine_heads(cx, sm, nst, base, gpt, tag)) dead = true;
            } else if (rows) {
                // q 0: x(l) = x1(l-1) + down(l-1); q 2: x1 = x + o_proj
                const unsigned long long* src =
                    q == 2 ? acc_ptr(a, epoch, l, MG_ACC_X1) : (l > 0 ? acc_ptr(a, epoch, l - 1, MG_ACC_X2) : nullptr);
                const int sp = q == 2 ? 1 : 2;  // tile counts: o_proj / down
                if (src) hint_acc(cx, src + (size_t)(a.ph[sp == 1 ? 1 : 3].tiles - 1) * 16 + 15,
                                  ms->tcount[sp][a.ph[sp == 1 ? 1 : 3].tiles - 1]);
                // (a failure seen during the hint makes the residual's polls return at once)
                if (residual_stats(cx, sm, a, src, ms->tcount[sp], q == 0 ? ln1 : ln2, F16)) dead = true;
            } else {
                // q 3: the SwiGLU outputs of this CTA's down range (tagged words, 4 per item)
                if (tid == 0) {
                    const uint64_t* hp = hb + (size_t)(B - 1) * a.FF + a.FF - 1;
                    if ((uint32_t)(ldr64(hp) >> 32) != tag) poll(cx, hp, tag);
                }
                if (check()) break;
                for (int e = tid; e < nst * 16 * B; e += MG_CT) {
                    const int qq = divB(e, ms->bm), b = e - qq * B, si = qq >> 4, k4 = qq & 15;
                    const int kg = si + base < gpt ? si + base : si + base - gpt;
                    const uint64_t* src = hb + (size_t)b * a.FF + kg * 64 + k4 * 4;
                    uint16_t* dst = sm.sT + (si * 64 + k4 * 4) * B + b;
                    const uint4 v0 = ldcg16(src), v1 = ldcg16(src + 2);
                    // the low half of each word is a bf16 bit pattern
                    if (v0.y == tag && v0.w == tag && v1.y == tag && v1.w == tag) {
                        dst[0] = (uint16_t)v0.x;
                        dst[B] = (uint16_t)v0.z;
                        dst[2 * B] = (uint16_t)v1.x;
                        dst[3 * B] = (uint16_t)v1.z;
                    } else {
                        poll4_bf16(src, dst, B, tag, cx.fail, a.err);
                    }
                }
                check();
            }
            // every branch above ended with a failure-reducing barrier
            if (dead) break;
            MG_STAMP(1 + 2 * q)
            sm.so = 10 + 7 * q;
            stage<F16, TR>(sm, nst, B, H, rows ? 0 : 1, q == 0 ? ln1 : ln2);
            const int which = q == 0 ? MG_ACC_QKV : (q == 1 ? MG_ACC_X1 : MG_ACC_X2);
            gemv_phase<FMT, TR>(cx, sm, q, cslot, cpar, ring, full, empty, base, rows, q == 2 ? OUT_GLU : OUT_ACC,
                            q == 2 ? nullptr : acc_ptr(a, epoch, l, which), hb, tag);
            cons += ms->nsc[q];
            cslot += ms->nsc[q];
            while (cslot >= a.nslots) {
                cslot -= a.nslots;
                cpar ^= 1u;
            }
            if (check()) break;
            MG_STAMP(2 + 2 * q)
        }
        // release the layer's parameter block to the producer
        if (!dead && tid == 0) mbar_arrive(&lp_empty[l & 1]);
    }
#undef MG_STAMP
    // ---------------- final norm + stop head (CTA b handles row b) ----------------
    if (!dead && c < B) {
        const unsigned long long* src = acc_ptr(a, epoch, a.layers - 1, MG_ACC_X2);
        hint_acc(cx, src + (size_t)(a.ph[3].tiles - 1) * 16 + 15, ms->tcount[2][a.ph[3].tiles - 1]);
        if (!check()) {
            residual_stats(cx, sm, a, src, ms->tcount[2], a.norm, false);
            const int b = c, warp = tid >> 5, lane = tid & 31;
            const float inv = ms->inv[b];
            uint16_t* ob = a.out_cell ? *a.out_cell : nullptr;
            uint16_t* oo = ob ? ob + ((size_t)ms->step * B + b) * H : nullptr;
            float l0 = 0.f, l1 = 0.f;
            for (int f = tid; f < H; f += MG_CT) {
                const float zf = rb(bf2f(a.norm[f]) * rb(bf2f(sm.sX[b * H + f]) * inv));
                const uint16_t zb = f2bf(zf);
                a.z[(size_t)b * H + f] = zb;
                a.feed[(size_t)b * H + f] = zb;
                if (oo) oo[f] = zb;
                l0 += bf2f(a.stop_w[f]) * zf;
                l1 += bf2f(a.stop_w[H + f]) * zf;
            }
            l0 = warp_sum(l0);
            l1 = warp_sum(l1);
            if (lane == 0) {
                ms->red[warp] = l0;
                ms->red[MG_CWARPS + warp] = l1;
            }
            cbar();
            if (tid == 0) {
                float s0 = 0.f, s1 = 0.f;
                for (int w = 0; w < MG_CWARPS; w++) {
                    s0 += ms->red[w];
                    s1 += ms->red[MG_CWARPS + w];
                }
                s0 = rb(s0 + bf2f(a.stop_b[0]));
                s1 = rb(s1 + bf2f(a.stop_b[1]));
                const float m = fmaxf(s0, s1), e0 = expf(s0 - m), e1 = expf(s1 - m);
                const float pr = e1 / (e0 + e1);
                a.stop[b] = pr;
                float* sb = a.stop_cell ? *a.stop_cell : nullptr;
                if (sb) sb[(size_t)ms->step * B + b] = pr;
            }
        }
    }
    // ---------------- wind-down ----------------
    if (dead || *(volatile int*)&ms->fail) {
        // record the failure, then wait (bounded) for this CTA's copies in flight
        if (tid == 0) {
            atomicCAS(a.err, 0, ms->fail ? ms->fail : 4);
            const long long t0 = clock64();
            while (!*(volatile int*)&ms->prod_done && clock64() - t0 < MG_TIMEOUT) {
            }
            const int issued = *(volatile int*)&ms->issued;
            for (int sc = cons; sc < issued; sc++) mbar_wait(&full[sc % a.nslots], (sc / a.nslots) & 1);
            for (int l = lp_used; l < a.layers && l < lp_used + 2; l++) mbar_wait(&lp_full[l & 1], (l >> 1) & 1);
            if (ms->att_inflight) mbar_wait(&ms->att_bar, ms->att_uses & 1u);  // an attention item's page copies
        }
        return;
    }
    if (c == 0 && tid == 0) {
        // every CTA read the epoch and positions before contributing to the
        // last layer, which this CTA waited for
        a.counter[0] = (int)epoch;
        a.counter[1] = ms->step + 1;
        for (int b = 0; b < B; b++) a.seq_len[ms->seq[b]] += 1;
    }
}

}  // namespace

int mega_smem_bytes(int nslots, int slot_bytes, int H, int lp_bytes) { return smem_map(nslots, slot_bytes, H, lp_bytes).total; }

cudaError_t launch_mega(const MegaDev& a, int smem, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.C);
    cfg.blockDim = dim3(MG_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaError_t e;
    auto go = [&](auto kern) {
        cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        return r == cudaSuccess ? cudaLaunchKernelEx(&cfg, kern, a) : r;
    };
    const bool tr = a.trace != nullptr;
    if (a.fmt == 4) e = tr ? go(mega_kernel<4, true>) : go(mega_kernel<4, false>);
    else if (a.fmt == 8) e = tr ? go(mega_kernel<8, true>) : go(mega_kernel<8, false>);
    else e = tr ? go(mega_kernel<16, true>) : go(mega_kernel<16, false>);
    return e;
}

}  // namespace ming
