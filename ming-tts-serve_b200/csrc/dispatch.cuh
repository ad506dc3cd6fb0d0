// dispatch.cuh — internal: picks the linear kernel for a packed weight and a
// row count (decode-batch linear, tiled mma.sync linears, staged fragments,
// tcgen05 linear) and launches it on a stream. Shared by the translation
// units that run linears (runtime.cu, vae.cu).
#pragma once

#include <algorithm>
#include <cstdlib>
#include <string>
#include <type_traits>

#include "bulk.cuh"
#include "runtime.h"
#include "tcgen05.cuh"

namespace ming {
namespace rt {

template <int FMT, int NT, class Pro, class Epi>
void launch_lin_t(const PackedW& W, const Pro& p, const Epi& e, int rows, cudaStream_t s) {
    static unsigned attr_devices = 0;  // bit d: attribute set on device d
    constexpr int smem = LinSmem<NT>::TOTAL;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_devices & (1u << (dev & 31)))) {
        cudaFuncSetAttribute(linear_kernel<FMT, NT, Pro, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        attr_devices |= 1u << (dev & 31);
    }
    dim3 grid(W.ntiles, (rows + 8 * NT - 1) / (8 * NT));
    linear_kernel<FMT, NT, Pro, Epi><<<grid, LIN_THREADS, smem, s>>>(W, p, e, rows);
}

template <int FMT, int NT, int T, class Epi>
void launch_lin_frag(const PackedW& W, const LinScratch& sc, const Epi& e, int rows, cudaStream_t s) {
    static unsigned attr_devices = 0;  // bit d: attribute set on device d
    constexpr int smem = LinSmem<NT>::B_BYTES + LinSmem<NT>::YS_BYTES + LinSmem<NT>::RED_BYTES;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_devices & (1u << (dev & 31)))) {
        cudaFuncSetAttribute(linear_frag_kernel<FMT, NT, T, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        attr_devices |= 1u << (dev & 31);
    }
    dim3 grid((W.ntiles + T - 1) / T, (rows + 8 * NT - 1) / (8 * NT));
    linear_frag_kernel<FMT, NT, T, Epi><<<grid, LIN_THREADS, smem, s>>>(W, sc, e, rows);
}

// More than 8 rows: the prologue runs once into the context's staging
// scratch, then CTAs of up to 4 tiles consume it (4 when that still gives
// every SM several CTAs).
template <int FMT, int NT, class Pro, class Epi>
void launch_lin_staged(const PackedW& W, const LinScratch& sc, const Pro& p, const Epi& e, int rows, cudaStream_t s) {
    dim3 sg((rows + 7) / 8, (W.K + STAGE_KC - 1) / STAGE_KC);
    stage_frag_kernel<FMT != 16, Pro><<<sg, LIN_THREADS, 0, s>>>(p, rows, W.K, sc, FMT != 16);
    const long ctas = (long)W.ntiles * ((rows + 8 * NT - 1) / (8 * NT));
    if (ctas >= 4L * sc.sms) launch_lin_frag<FMT, NT, 4>(W, sc, e, rows, s);
    else launch_lin_frag<FMT, NT, 1>(W, sc, e, rows, s);
}

// F16: f16 operands (the prefill copies of quantized weights), else bf16
template <int N, bool F16, class Pro, class Epi>
void launch_tc_n(const PackedW& W, const LinScratch& sc, const Pro& p, const Epi& e, int rows, int ks, cudaStream_t s) {
    const int KT = W.tck;  // K of the weight blocks (the rows are staged over it)
    static unsigned attr_devices = 0;  // bit d: attribute set on device d
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr int smax = N <= 128 ? TcSmem<N>::TOTAL_KS : TcSmem<N>::TOTAL;
    if (!(attr_devices & (1u << (dev & 31)))) {
        cudaFuncSetAttribute(tc_linear_kernel<N, Epi, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax);
        attr_devices |= 1u << (dev & 31);
    }
    if (N > 128) ks = 1;  // no room for the partial sums beside the 256-row stages
    uint8_t* xs = reinterpret_cast<uint8_t*>(sc.frag);
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    {
        cudaLaunchConfig_t sg = {};
        sg.gridDim = dim3((rows + 7) / 8, (KT + STAGE_KC - 1) / STAGE_KC);
        sg.blockDim = dim3(LIN_THREADS);
        sg.stream = s;
        sg.attrs = pdl;
        sg.numAttrs = 1;
        cudaLaunchKernelEx(&sg, stage_rows_kernel<N, Pro, F16>, p, rows, KT, xs, (float*)sc.post);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(W.ntiles / 8 * ks), (unsigned)((rows + N - 1) / N));
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = ks > 1 ? (size_t)TcSmem<N>::TOTAL_KS : (size_t)TcSmem<N>::TOTAL;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0] = pdl[0];
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = (unsigned)ks;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = ks > 1 ? 2 : 1;
    cudaLaunchKernelEx(&cfg, tc_linear_kernel<N, Epi, F16>, W.tc, KT, (const uint8_t*)xs, (const float*)sc.post, e, rows, ks);
}

// bf16 weights, 64+ rows: the tcgen05 linear with the widest row block that
// still gives ~96 CTAs; when even 64-row blocks leave fewer than half the SMs
// a CTA, the K groups are split over a cluster of up to 8 CTAs (at least 12
// groups each).
template <bool F16, class Pro, class Epi>
void launch_tc(const PackedW& W, const LinScratch& sc, const Pro& p, const Epi& e, int rows, cudaStream_t s) {
    const int mt = W.ntiles / 8;
    if (mt * ((rows + 255) / 256) >= 96) launch_tc_n<256, F16>(W, sc, p, e, rows, 1, s);
    else if (mt * ((rows + 127) / 128) >= 96) launch_tc_n<128, F16>(W, sc, p, e, rows, 1, s);
    else {
        const int ctas = mt * ((rows + 63) / 64);
        int ks = 1;
        if (2 * ctas <= sc.sms) ks = std::max(1, std::min({8, sc.sms / ctas, W.tck / 64 / 12}));
        launch_tc_n<64, F16>(W, sc, p, e, rows, ks, s);
    }
}

inline bool bulk_enabled() {
    static const bool on = [] {
        const char* v = getenv("MING_BULK");
        return !(v && std::string(v) == "0");
    }();
    return on;
}

// MING_TC_COPIES=0: no f16 prefill copies of quantized linears (their
// prefill then stays on the mma.sync kernels)
inline bool tc_copies_enabled() {
    static const bool on = [] {
        const char* v = getenv("MING_TC_COPIES");
        return !(v && std::string(v) == "0");
    }();
    return on;
}

inline bool tc_enabled() {
    static const bool on = [] {
        const char* v = getenv("MING_TC");
        return !(v && std::string(v) == "0");
    }();
    return on;
}

template <int FMT, class Pro, class Epi>
void launch_lin_f(const LinScratch& sc, const PackedW& W, const Pro& p, const Epi& e, int rows, cudaStream_t s) {
    const bool staged = sc.frag && rows <= sc.rows && W.K <= sc.K;
    // bf16 weights from 64 rows; quantized weights (their f16 prefill copy,
    // f16 rows) above 64 rows, so decode batches up to 64 rows keep the
    // 4/8-bit bytes
    if (staged && (FMT == 16 ? rows >= 64 : rows > 64) && W.tc && W.tck <= sc.K && tc_enabled()) {
        if (W.tck == W.K) launch_tc<FMT != 16>(W, sc, p, e, rows, s);
        else launch_tc<FMT != 16>(W, sc, ProTwice<Pro>{p, W.K}, e, rows, s);
        return;
    }
    // up to 64 rows of plain, RMS-normed or LayerNorm-modulated inputs: bulk.cuh
    if constexpr (std::is_same_v<Pro, ProRms> || std::is_same_v<Pro, ProPlain> || std::is_same_v<Pro, ProLnMod>) {
        if (rows <= 64 && sc.err && bulk_enabled()) {
            if constexpr (std::is_same_v<Pro, ProRms>) {
                if (p.K == W.K && p.ld % 8 == 0 &&
                    launch_bulk<FMT, BK_RMS>(W, BulkIn{p.x, p.unit ? nullptr : p.nw, p.ld, p.eps, sc.err, sc.trace}, e, rows,
                                             sc.sms, s))
                    return;
            } else if constexpr (std::is_same_v<Pro, ProLnMod>) {
                const bool al = ((uintptr_t)p.shift % 16 == 0) && ((uintptr_t)p.scale % 16 == 0);
                if (p.K == W.K && p.ld % 8 == 0 && p.mod_ld % 8 == 0 && al &&
                    launch_bulk<FMT, BK_LNMOD>(W,
                                               BulkIn{p.x, nullptr, p.ld, 0.f, sc.err, sc.trace, p.shift, p.scale, p.mod_ld,
                                                      p.rows_per_cond},
                                               e, rows, sc.sms, s))
                    return;
            } else {
                if (p.ld % 8 == 0 &&
                    launch_bulk<FMT, BK_PLAIN>(W, BulkIn{p.x, nullptr, p.ld, 0.f, sc.err, sc.trace}, e, rows, sc.sms, s))
                    return;
            }
        }
    }
    if (rows <= 8) launch_lin_t<FMT, 1>(W, p, e, rows, s);
    else if (rows <= 16) {
        if (staged) launch_lin_staged<FMT, 2>(W, sc, p, e, rows, s);
        else launch_lin_t<FMT, 2>(W, p, e, rows, s);
    } else {
        if (staged) launch_lin_staged<FMT, 4>(W, sc, p, e, rows, s);
        else launch_lin_t<FMT, 4>(W, p, e, rows, s);
    }
}

template <class Pro, class Epi>
void run_linear(ming_ctx* c, const PackedW& W, const Pro& p, const Epi& e, int rows, cudaStream_t s) {
    if (rows <= 0) return;
    LinScratch sc = c->lin;
    sc.trace = ktrace_slot(c);
    if (W.fmt == 4) launch_lin_f<4>(sc, W, p, e, rows, s);
    else if (W.fmt == 8) launch_lin_f<8>(sc, W, p, e, rows, s);
    else launch_lin_f<16>(sc, W, p, e, rows, s);
}

}  // namespace rt
}  // namespace ming
