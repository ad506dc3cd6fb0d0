// pack.cpp — repacks reference-layout weights (bf16 [out][in] or MLX affine
// 4/8-bit) into the kernels' tile layout (see pack.h).
#include "pack.h"

#include <cstring>

namespace ming {

static inline float h_bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Integer code of element k of row `row` in MLX packing: word k/(32/bits),
// bits [bits*(k%per), +bits).
static inline uint32_t code_at(const LinearSrc& s, int row, int k) {
    const int per = 32 / s.fmt;
    const uint32_t w = s.q[(int64_t)row * (s.in / per) + k / per];
    return (w >> (s.fmt * (k % per))) & ((1u << s.fmt) - 1u);
}

std::string pack_tiles(const std::vector<LinearSrc>& srcs, const std::vector<RowRef>& rows, int fmt, int K,
                       std::vector<uint8_t>& out, std::vector<float>& bias_out) {
    if (rows.size() % 16) return "pack: row count is not a multiple of 16";
    if (K % 64) return "pack: K is not a multiple of 64";
    for (const auto& s : srcs) {
        if (s.fmt != fmt) return "pack: mixed weight formats in one packed linear";
        if (s.in != K) return "pack: source in-dimension differs from K";
        if (fmt != 16 && s.group != 64) return "pack: only group size 64 is supported";
        if (fmt == 16 && !s.w) return "pack: missing bf16 weight";
        if (fmt != 16 && (!s.q || !s.scales || !s.biases)) return "pack: missing quantized weight, scales or biases";
    }
    const int ntiles = (int)rows.size() / 16, ng = K / 64, cb = chunk_bytes(fmt);
    out.assign((size_t)ntiles * ng * cb, 0);
    bias_out.assign(rows.size(), 0.0f);
    for (size_t i = 0; i < rows.size(); i++) {
        const RowRef& r = rows[i];
        if (r.src >= 0 && srcs[r.src].bias) bias_out[i] = h_bf2f(srcs[r.src].bias[r.row]);
    }
    for (int t = 0; t < ntiles; t++) {
        for (int g = 0; g < ng; g++) {
            uint8_t* ch = out.data() + ((size_t)t * ng + g) * cb;
            for (int lane = 0; lane < 32; lane++) {
                const int gr = lane >> 2, tq = lane & 3;
                for (int ks = 0; ks < 4; ks++) {
                    const int kb = g * 64 + ks * 16;
                    // (row-in-tile, k) of the 8 fragment elements in register order a0..a3 (lo, hi)
                    const int er[8] = {gr, gr, gr + 8, gr + 8, gr, gr, gr + 8, gr + 8};
                    const int ek[8] = {kb + 2 * tq, kb + 2 * tq + 1, kb + 2 * tq, kb + 2 * tq + 1,
                                       kb + 2 * tq + 8, kb + 2 * tq + 9, kb + 2 * tq + 8, kb + 2 * tq + 9};
                    if (fmt == 16) {
                        uint16_t v[8];
                        for (int e = 0; e < 8; e++) {
                            const RowRef& rr = rows[t * 16 + er[e]];
                            v[e] = rr.src < 0 ? 0 : srcs[rr.src].w[(int64_t)rr.row * K + ek[e]];
                        }
                        std::memcpy(ch + ((size_t)ks * 32 + lane) * 16, v, 16);
                    } else if (fmt == 4) {
                        // nibble i: (n0,n4)=a0, (n1,n5)=a1, (n2,n6)=a2, (n3,n7)=a3
                        static const int slot[8] = {0, 4, 1, 5, 2, 6, 3, 7};
                        uint32_t w = 0;
                        for (int e = 0; e < 8; e++) {
                            const RowRef& rr = rows[t * 16 + er[e]];
                            const uint32_t c = rr.src < 0 ? 0 : code_at(srcs[rr.src], rr.row, ek[e]);
                            w |= c << (4 * slot[e]);
                        }
                        std::memcpy(ch + (size_t)lane * 16 + ks * 4, &w, 4);
                    } else {
                        // w0 bytes: A[g][2t], A[g][2t+1], A[g+8][2t], A[g+8][2t+1]; w1 the same at k+8
                        uint32_t w0 = 0, w1 = 0;
                        for (int e = 0; e < 8; e++) {
                            const RowRef& rr = rows[t * 16 + er[e]];
                            const uint32_t c = rr.src < 0 ? 0 : code_at(srcs[rr.src], rr.row, ek[e]);
                            if (e < 4) w0 |= c << (8 * e);
                            else w1 |= c << (8 * (e - 4));
                        }
                        // [half = ks/2][lane][4 words]: words (w0,w1) of ks even, then odd
                        uint8_t* p = ch + ((size_t)(ks >> 1) * 32 + lane) * 16 + (ks & 1) * 8;
                        std::memcpy(p, &w0, 4);
                        std::memcpy(p + 4, &w1, 4);
                    }
                }
            }
            if (fmt != 16) {
                uint16_t* sc = reinterpret_cast<uint16_t*>(ch + (fmt == 4 ? 512 : 1024));
                for (int gr = 0; gr < 8; gr++) {
                    for (int h = 0; h < 2; h++) {
                        const RowRef& rr = rows[t * 16 + gr + 8 * h];
                        uint16_t s = 0, b = 0;
                        if (rr.src >= 0) {
                            const LinearSrc& src = srcs[rr.src];
                            s = src.scales[(int64_t)rr.row * ng + g];
                            b = src.biases[(int64_t)rr.row * ng + g];
                        }
                        sc[gr * 4 + 2 * h] = s;
                        sc[gr * 4 + 2 * h + 1] = b;
                    }
                }
            }
        }
    }
    return "";
}

}  // namespace ming
