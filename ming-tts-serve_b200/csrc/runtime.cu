// runtime.cu — the context behind include/ming_cuda.h: weight staging and
// repacking, the paged KV allocator, captured decode graphs, the flow head.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <memory>
#include <string>
#include <type_traits>
#include <vector>

#include "runtime.h"
#include "dispatch.cuh"
#include "bulk.cuh"
#include "dit.cuh"
#include "lm.cuh"
#include "mega.cuh"
#include "tcgen05.cuh"
#include "pack.h"

using namespace ming;
using namespace ming::rt;

// ---------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------

static thread_local std::string g_err;

int ming::rt::fail(int code, const std::string& m) {
    g_err = m;
    return code;
}

// ---------------------------------------------------------------------
// linear launch dispatch
// ---------------------------------------------------------------------

namespace ming {
namespace rt {

// Dequantizes every tile of a packed linear to f32 [ntiles*16][K] (the
// kernels' unpack functions; used by ming_cuda_unpack_linear).
__global__ void unpack_tiles_kernel(PackedW W, float* out) {
    const int tile = blockIdx.x, gi = blockIdx.y, lane = threadIdx.x;
    const int ng = W.K / 64, cb = chunk_b(W.fmt);
    const uint8_t* ch = W.tiles + ((size_t)tile * ng + gi) * cb;
    const int g = lane >> 2, t = lane & 3;
    float s_lo = 1.f, b_lo = 0.f, s_hi = 1.f, b_hi = 0.f;
    if (W.fmt != 16) {
        const uint2 sc = *reinterpret_cast<const uint2*>(ch + (W.fmt == 4 ? 512 : 1024) + g * 8);
        s_lo = __uint_as_float(sc.x << 16);
        b_lo = __uint_as_float(sc.x & 0xffff0000u);
        s_hi = __uint_as_float(sc.y << 16);
        b_hi = __uint_as_float(sc.y & 0xffff0000u);
    }
    for (int ks = 0; ks < 4; ks++) {
        uint32_t a[4];
        if (W.fmt == 16) {
            const uint4 w = *reinterpret_cast<const uint4*>(ch + ((size_t)ks * 32 + lane) * 16);
            a[0] = w.x; a[1] = w.y; a[2] = w.z; a[3] = w.w;
        } else if (W.fmt == 4) {
            const uint32_t w = reinterpret_cast<const uint32_t*>(ch + (size_t)lane * 16)[ks];
            dq4(w, a);
        } else {
            const uint32_t* p = reinterpret_cast<const uint32_t*>(ch + ((size_t)(ks >> 1) * 32 + lane) * 16 + (ks & 1) * 8);
            dq8(p[0], p[1], a);
        }
        const int k0 = gi * 64 + ks * 16 + 2 * t;
        const int rr[4] = {g, g + 8, g, g + 8};
        const int kk[4] = {k0, k0, k0 + 8, k0 + 8};
        for (int i = 0; i < 4; i++) {
            float lo, hi;
            if (W.fmt == 16) {
                const float2 v = unpack_bf16x2(a[i]);
                lo = v.x;
                hi = v.y;
            } else {
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&a[i]));
                const float s = rr[i] < 8 ? s_lo : s_hi, b = rr[i] < 8 ? b_lo : b_hi;
                lo = s * v.x + b;
                hi = s * v.y + b;
            }
            float* o = out + (size_t)(tile * 16 + rr[i]) * W.K + kk[i];
            o[0] = lo;
            o[1] = hi;
        }
    }
}

// Writes K/V rows [n][64] of one layer into the paged pool through the block
// table and kv_index, the same index function the decode kernels append
// with (ming_cuda_kv_write). Grid (n, kv_heads, K|V), 64 threads: one value each.
__global__ void kv_write_kernel(KvDev kv, int seq, int layer, int pos0, int n, const uint16_t* k, const uint16_t* v) {
    const int j = blockIdx.x, h = blockIdx.y, which = blockIdx.z, d = threadIdx.x, pos = pos0 + j;
    const int page = kv.bt[(size_t)seq * kv.bt_ld + pos / PAGE];
    const uint16_t* src = which ? v : k;
    kv.pool[kv_index(kv, page, layer, which, h, pos % PAGE) + d] = src[((size_t)h * n + j) * HD + d];
}

// ---------------------------------------------------------------------
// staging helpers
// ---------------------------------------------------------------------

const HostTensor* find(ming_ctx* c, const std::string& n) {
    auto it = c->staged.find(n);
    return it == c->staged.end() ? nullptr : &it->second;
}
const HostTensor* find_staged(ming_ctx* c, const std::string& n) { return find(c, n); }

int lin_src(ming_ctx* c, const std::string& prefix, LinearSrc& s, bool want_bias) {
    const HostTensor* w = find(c, prefix + ".weight");
    if (!w) return fail(MING_ERR_MISSING, "missing weight " + prefix + ".weight");
    const HostTensor* sc = find(c, prefix + ".scales");
    const HostTensor* bi = find(c, prefix + ".biases");
    if (w->shape.size() != 2) return fail(MING_ERR_INVALID, prefix + ".weight is not 2-D");
    s = LinearSrc{};
    s.out = (int)w->shape[0];
    if (sc) {
        if (!bi) return fail(MING_ERR_MISSING, "missing " + prefix + ".biases");
        if (w->dtype != MING_DTYPE_U32 || sc->dtype != MING_DTYPE_BF16 || bi->dtype != MING_DTYPE_BF16)
            return fail(MING_ERR_INVALID, prefix + ": quantized weight must be U32 with BF16 scales/biases");
        if (sc->shape.size() != 2 || sc->shape[0] != s.out || bi->shape != sc->shape)
            return fail(MING_ERR_INVALID, prefix + ": scales/biases shape mismatch");
        s.group = c->cfg.group_size;
        s.in = (int)sc->shape[1] * s.group;
        const int64_t words = w->shape[1];
        if (s.in == 0 || (words * 32) % s.in) return fail(MING_ERR_INVALID, prefix + ": cannot infer bit width");
        s.fmt = (int)(words * 32 / s.in);
        if (s.fmt != 4 && s.fmt != 8) return fail(MING_ERR_INVALID, prefix + ": only 4/8-bit quantization is supported");
        s.q = reinterpret_cast<const uint32_t*>(w->data.data());
        s.scales = reinterpret_cast<const uint16_t*>(sc->data.data());
        s.biases = reinterpret_cast<const uint16_t*>(bi->data.data());
    } else {
        if (w->dtype != MING_DTYPE_BF16) return fail(MING_ERR_INVALID, prefix + ".weight must be BF16 (or U32 + scales)");
        s.fmt = 16;
        s.in = (int)w->shape[1];
        s.w = reinterpret_cast<const uint16_t*>(w->data.data());
    }
    if (want_bias) {
        const HostTensor* b = find(c, prefix + ".bias");
        if (!b) return fail(MING_ERR_MISSING, "missing " + prefix + ".bias");
        if (b->dtype != MING_DTYPE_BF16 || b->data.size() != (size_t)s.out * 2)
            return fail(MING_ERR_INVALID, prefix + ".bias must be BF16 [out]");
        s.bias = reinterpret_cast<const uint16_t*>(b->data.data());
    }
    return MING_OK;
}

int upload_packed(ming_ctx* c, const std::vector<LinearSrc>& srcs, const std::vector<std::string>& names,
                  const std::vector<RowRef>& rows, PackedLin& pl) {
    const int fmt = srcs[0].fmt, K = srcs[0].in;
    std::vector<uint8_t> tiles;
    std::vector<float> bias;
    std::string e = pack_tiles(srcs, rows, fmt, K, tiles, bias);
    if (!e.empty()) return fail(MING_ERR_INVALID, names[0] + ": " + e);
    int rc = MING_OK;
    uint8_t* dt = c->mem.alloc<uint8_t>(tiles.size(), &rc);
    if (!dt) return rc;
    float* db = c->mem.alloc<float>(bias.size(), &rc);
    if (!db) return rc;
    CK(cudaMemcpy(dt, tiles.data(), tiles.size(), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(db, bias.data(), bias.size() * 4, cudaMemcpyHostToDevice));
    pl.w.tiles = dt;
    pl.w.bias = db;
    pl.w.ntiles = (int)rows.size() / 16;
    pl.w.K = K;
    pl.w.fmt = fmt;
    if (fmt == 16 && pl.w.ntiles % 8 == 0 && K % 64 == 0) {
        // the tcgen05 linear's weight blocks (same bytes, swizzled shared-memory order)
        uint8_t* tc = c->mem.alloc<uint8_t>(tiles.size(), &rc);
        if (!tc) return rc;
        tc_swizzle_kernel<<<dim3(pl.w.ntiles / 8, K / 64), TC_THREADS>>>(dt, K / 64, tc);
        CK(cudaGetLastError());
        pl.w.tc = tc;
        pl.w.tck = K;
    } else if ((fmt == 4 || fmt == 8) && pl.w.ntiles % 8 == 0 && K % 64 == 0 && c->cfg.max_prefill > 64 && tc_copies_enabled()) {
        // the prefill copy: f16 hi | lo weight blocks dequantized once at load,
        // so chunks of more than 64 rows run on the tcgen05 linear (4 bytes
        // per weight in HBM beside the packed tiles)
        uint8_t* tc = c->mem.alloc<uint8_t>((size_t)pl.w.ntiles * 16 * K * 4, &rc);
        if (!tc) return rc;
        tc_swizzle_dq_kernel<<<dim3(pl.w.ntiles / 8, K / 64), TC_THREADS>>>(dt, K / 64, fmt, tc);
        CK(cudaGetLastError());
        pl.w.tc = tc;
        pl.w.tck = 2 * K;
    }
    pl.src_names = names;
    pl.rows = rows;
    for (auto& s : srcs) {
        pl.src_out.push_back(s.out);
        pl.src_in.push_back(s.in);
    }
    c->all_lins.push_back(&pl);
    return MING_OK;
}

// True when a staged bf16 gain vector holds only 1.0.
bool unit_gains(ming_ctx* c, const std::string& name) {
    auto it = c->staged.find(name);
    if (it == c->staged.end() || it->second.dtype != MING_DTYPE_BF16) return false;
    const auto& d = it->second.data;
    for (size_t i = 0; i + 1 < d.size(); i += 2)
        if (d[i] != 0x80 || d[i + 1] != 0x3F) return false;
    return !d.empty();
}

// Plain row order: tile row r -> source row 16t + r (zero rows past `out`).
int pack_plain(ming_ctx* c, const std::string& prefix, bool bias, PackedLin& pl, int* out_dim) {
    LinearSrc s;
    int rc = lin_src(c, prefix, s, bias);
    if (rc) return rc;
    if (out_dim) *out_dim = s.out;
    std::vector<RowRef> rows(((s.out + 15) / 16) * 16);
    for (size_t i = 0; i < rows.size(); i++) rows[i] = (int)i < s.out ? RowRef{0, (int)i} : RowRef{-1, 0};
    return upload_packed(c, {s}, {prefix + ".weight"}, rows, pl);
}

int upload_raw(ming_ctx* c, const std::string& name, int dtype, int64_t count, void** out) {
    const HostTensor* t = find(c, name);
    if (!t) return fail(MING_ERR_MISSING, "missing weight " + name);
    const size_t esz = dtype == MING_DTYPE_BF16 ? 2 : 4;
    if (t->dtype != dtype || t->data.size() != (size_t)count * esz)
        return fail(MING_ERR_INVALID, name + ": unexpected dtype or size");
    int rc = MING_OK;
    uint8_t* d = c->mem.alloc<uint8_t>(t->data.size(), &rc);
    if (!d) return rc;
    CK(cudaMemcpy(d, t->data.data(), t->data.size(), cudaMemcpyHostToDevice));
    *out = d;
    return MING_OK;
}

// DiT q|k|v with neighbour-interleaved rows (rotary pairs in one thread).
int pack_dit_qkv(ming_ctx* c, const std::string& pre, PackedLin& pl, int H) {
    LinearSrc s[3];
    const char* nm[3] = {".attn.to_q", ".attn.to_k", ".attn.to_v"};
    for (int i = 0; i < 3; i++) {
        int rc = lin_src(c, pre + nm[i], s[i], true);
        if (rc) return rc;
        if (s[i].out != H) return fail(MING_ERR_INVALID, pre + nm[i] + ": wrong out dim");
    }
    std::vector<RowRef> rows;
    for (int b = 0; b < 3; b++)
        for (int lt = 0; lt < H / 16; lt++)
            for (int r = 0; r < 16; r++) rows.push_back({b, r < 8 ? lt * 16 + 2 * r : lt * 16 + 2 * (r - 8) + 1});
    return upload_packed(c, {s[0], s[1], s[2]}, {pre + nm[0] + ".weight", pre + nm[1] + ".weight", pre + nm[2] + ".weight"},
                         rows, pl);
}

int load_dit_blocks(ming_ctx* c, const std::string& prefix, int nblocks, int H, bool adaln, std::vector<DitBlockW>& out) {
    out.resize(nblocks);
    for (int i = 0; i < nblocks; i++) {
        const std::string pre = prefix + ".blocks." + std::to_string(i);
        DitBlockW& b = out[i];
        int rc;
        if (adaln) {
            if ((rc = pack_plain(c, pre + ".adaLN_modulation.1", true, b.ada))) return rc;
        } else {
            if ((rc = upload_raw(c, pre + ".norm1.weight", MING_DTYPE_BF16, H, (void**)&b.norm1))) return rc;
            if ((rc = upload_raw(c, pre + ".norm2.weight", MING_DTYPE_BF16, H, (void**)&b.norm2))) return rc;
        }
        if ((rc = pack_dit_qkv(c, pre, b.qkv, H))) return rc;
        if ((rc = pack_plain(c, pre + ".attn.to_out.0", true, b.o))) return rc;
        if ((rc = pack_plain(c, pre + ".mlp.ff.0.0", true, b.ff1))) return rc;
        if ((rc = pack_plain(c, pre + ".mlp.ff.2", true, b.ff2))) return rc;
    }
    return MING_OK;
}

// EPSS + sway flow schedule in bf16 (flowSchedule, src/ming_model.zig:1205-1215).
float h_rb(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    std::memcpy(&f, &u, 4);
    return f;
}
uint16_t h_f2bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void flow_schedule(float* t, float* dt, float* sq) {
    static const float sched[11] = {0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32};
    const float hh = h_rb(1.0f / 32.0f), hp = h_rb(3.14159265358979f / 2.0f);
    for (int i = 0; i <= 10; i++) {
        const float tt = h_rb(hh * h_rb(sched[i]));
        const float ct = h_rb(cosf(h_rb(hp * tt)));
        const float sw = h_rb(h_rb(ct - 1.0f) + tt);
        t[i] = h_rb(tt + h_rb(-1.0f * sw));
    }
    for (int i = 0; i < 10; i++) {
        dt[i] = h_rb(t[i + 1] - t[i]);
        sq[i] = h_rb(powf(fabsf(dt[i]), 0.5f));
    }
}

// Timestep embeddings of the 10 Euler steps (TimestepEmbedder,
// src/ming_model.zig:1064-1076; t_freq :966-975): sinusoid table on the
// host, the two linears + SiLU on the device.
int build_temb(ming_ctx* c, int freq_dim, int H) {
    float t[11];
    flow_schedule(t, c->flow_dt, c->flow_sq);
    const int half = freq_dim / 2;
    const float e = (float)(std::log(10000.0) / (double)(half - 1));
    std::vector<uint16_t> sc((size_t)10 * freq_dim);
    for (int r = 0; r < 10; r++) {
        const float ts = h_rb(h_rb(1000.0f) * t[r]);
        for (int j = 0; j < half; j++) {
            const float a = ts * std::exp((float)j * -e);
            sc[(size_t)r * freq_dim + j] = h_f2bf(std::sin(a));
            sc[(size_t)r * freq_dim + half + j] = h_f2bf(std::cos(a));
        }
    }
    int rc = MING_OK;
    uint16_t* d_sc = c->mem.alloc<uint16_t>(sc.size(), &rc);
    uint16_t* d_h0 = c->mem.alloc<uint16_t>((size_t)10 * H, &rc);
    c->temb = c->mem.alloc<uint16_t>((size_t)10 * H, &rc);
    if (rc) return rc;
    CK(cudaMemcpy(d_sc, sc.data(), sc.size() * 2, cudaMemcpyHostToDevice));
    run_linear(c, c->t_mlp0.w, ProPlain{d_sc, freq_dim, 0}, EpiAct{d_h0, nullptr, c->t_mlp0.w.bias, H, 2, H}, 10, c->stream);
    run_linear(c, c->t_mlp2.w, ProPlain{d_h0, H, 0}, EpiAct{c->temb, nullptr, c->t_mlp2.w.bias, H, 0, H}, 10, c->stream);
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
    return MING_OK;
}

int check_seq(ming_ctx* c, int s) {
    if (s < 0 || s >= (int)c->seqs.size() || !c->seqs[s].live) return fail(MING_ERR_INVALID, "invalid sequence id");
    return MING_OK;
}

// Makes sure positions [from, to) of sequence s have pages; uploads new
// block-table entries.
int ensure_pages(ming_ctx* c, int s, int from, int to) {
    if (to > c->cfg.max_ctx) return fail(MING_ERR_NOMEM, "sequence would exceed max_ctx positions");
    for (int p = from / PAGE; p < (to + PAGE - 1) / PAGE; p++) {
        int& e = c->bt_host[(size_t)s * c->bt_ld + p];
        if (e >= 0) continue;
        if (c->free_pages.empty()) return fail(MING_ERR_NOMEM, "KV page pool exhausted");
        e = c->free_pages.back();
        c->free_pages.pop_back();
        CK(cudaMemcpyAsync(c->bt + (size_t)s * c->bt_ld + p, &e, 4, cudaMemcpyHostToDevice, c->stream));
    }
    return MING_OK;
}

int copy_in(ming_ctx* c, void* dst, const void* src, size_t bytes, int kind) {
    if (bytes == 0) return MING_OK;
    CK(cudaMemcpyAsync(dst, src, bytes, kind == MING_PTR_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                       c->stream));
    return MING_OK;
}
int copy_out(ming_ctx* c, void* dst, const void* src, size_t bytes, int kind) {
    if (bytes == 0 || !dst) return MING_OK;
    CK(cudaMemcpyAsync(dst, src, bytes, kind == MING_PTR_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                       c->stream));
    return MING_OK;
}

constexpr int KT_SLOTS = 160, KT_CTAS = 1024;

long long* ktrace_slot(ming_ctx* c) {
    if (!c->ktrace || c->ktrace_used >= KT_SLOTS) return nullptr;
    return c->ktrace + (size_t)(c->ktrace_used++) * KT_CTAS * 8;
}

// The 24-layer step over `rows` rows whose row_seq/row_pos are on the device.
// Returns the first failed attention launch (the linears' launches are
// checked by the caller's cudaGetLastError).
cudaError_t enqueue_layers(ming_ctx* c, int rows, bool decode) {
    const ming_cfg& f = c->cfg;
    c->ktrace_used = 0;
    RowsDev rd{c->row_seq, c->row_pos};
    KvDev kv{c->pool, c->bt, c->bt_ld, f.layers, f.kv_heads};
    for (int l = 0; l < f.layers; l++) {
        auto& L = c->layers[l];
        run_linear(c, L.qkv.w, ProRms{c->x, L.ln1, f.hidden, f.hidden, f.rms_eps, 0, nullptr, L.ln1_unit},
                   EpiQKV{L.qkv.w.bias, c->q, kv, rd, l, f.heads, f.kv_heads, c->log2_theta}, rows, c->stream);
        AttnArgs aa{c->q, c->part, kv, rd, l, f.heads, f.kv_heads, c->nsplit, decode ? 1 : 0, c->att};
        aa.tmap = &c->kv_tmap;
        aa.err = c->dev_err;
        aa.trace = (long)aa.nsplit_max * aa.kv_heads * rows <= KT_CTAS ? ktrace_slot(c) : nullptr;
        cudaError_t e = launch_attn(aa, rows, c->stream);
        if (e == cudaSuccess && !attn_fused_combine(aa))
            e = launch_attn_combine(c->part, rd, c->nsplit, f.heads, c->att, rows, c->stream);
        if (e != cudaSuccess) return e;
        run_linear(c, L.o.w, ProPlain{c->att, f.heads * HD, 0},
                   EpiResidual{c->x, c->x1, nullptr, f.hidden}, rows, c->stream);
        run_linear(c, L.gu.w, ProRms{c->x1, L.ln2, f.hidden, f.hidden, f.rms_eps, 0, nullptr, L.ln2_unit}, EpiSwiGLU{c->h, f.ff}, rows,
                   c->stream);
        run_linear(c, L.down.w, ProPlain{c->h, f.ff, 0}, EpiResidual{c->x1, c->x, nullptr, f.hidden}, rows, c->stream);
    }
    return cudaSuccess;
}

StepDev step_dev(ming_ctx* c) {
    return StepDev{c->seq_len, c->row_seq, c->row_pos, c->step_counter, c->out_cell, c->stop_cell};
}

cudaError_t decode_enqueue(ming_ctx* c, int B) {
    if (c->mega_on && B <= MG_MAXB) {
        // one persistent launch per step: it reads the positions, bumps them,
        // and writes z, the fed-back input and the stop probabilities
        MegaDev a = c->mega;
        a.B = B;
        a.row_seq = c->row_seq;
        a.x_in = c->x;
        a.z = c->z;
        a.feed = c->x;
        a.stop = c->stop;
        return launch_mega(a, c->mega_smem, c->stream);
    }
    launch_step_begin(step_dev(c), B, c->stream);
    const cudaError_t le = enqueue_layers(c, B, true);
    launch_final(FinalArgs{c->x, c->norm, c->stop_w, c->stop_b, c->z, c->stop, c->x, step_dev(c), c->cfg.hidden, 0, 1,
                           c->cfg.rms_eps},
                 B, c->stream);
    return le;
}

// Decode graph for B rows: step_begin, layers, final (+ feedback into x).
int decode_graph(ming_ctx* c, int B, cudaGraphExec_t* out) {
    auto it = c->decode_graphs.find(B);
    if (it != c->decode_graphs.end()) {
        *out = it->second;
        return MING_OK;
    }
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const cudaError_t le = decode_enqueue(c, B);
    cudaError_t ce = cudaStreamEndCapture(c->stream, &g);
    if (le != cudaSuccess) {
        if (ce == cudaSuccess) cudaGraphDestroy(g);
        return fail(MING_ERR_CUDA, std::string("decode step launch: ") + cudaGetErrorString(le));
    }
    if (ce != cudaSuccess) return fail(MING_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
    cudaGraphExec_t ge;
    ce = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (ce != cudaSuccess) return fail(MING_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
    c->decode_graphs[B] = ge;
    *out = ge;
    return MING_OK;
}

// Plans the persistent decode kernel: per-phase group ranges of every CTA,
// per-tile contributor counts, counted fixed-point accumulators, buffers. Leaves it off when the device cannot co-schedule
// one CTA per SM (no cooperative launch) or MING_MEGA=0.
int setup_mega(ming_ctx* c) {
    const ming_cfg& f = c->cfg;
    const char* env = getenv("MING_MEGA");
    if (env && std::string(env) == "0") return MING_OK;
    int nsm = 0, coop = 0, optin = 0;
    CK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, c->device));
    CK(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, c->device));
    CK(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device));
    if (!coop) return MING_OK;
    const int H = f.hidden, fmt = f.weight_bits, cb = chunk_bytes(fmt);
    const int gps = fmt == 4 ? 14 : (fmt == 8 ? 7 : 4);
    const int slot = (gps * cb + 127) / 128 * 128;
    // per-layer parameter block: ln1 | ln2 (bf16) | q|k|v bias (f32), 16-byte multiple
    const int qkv_rows = (f.heads + 2 * f.kv_heads) * 64;
    const int lp_bytes = (4 * H + 4 * qkv_rows + 15) / 16 * 16;
    int nslots = 0;
    while (mega_smem_bytes(nslots + 1, slot, H, lp_bytes) <= optin) nslots++;
    MegaDev& a = c->mega;
    a = MegaDev{};
    const int tiles[MG_NPH] = {(f.heads + 2 * f.kv_heads) * 4, H / 16, f.ff / 8, H / 16};
    const int gpt[MG_NPH] = {H / 64, H / 64, H / 64, f.ff / 64};
    const int C = nsm;
    int rc = MING_OK;
    for (int p = 0; p < MG_NPH; p++) {
        const int G = tiles[p] * gpt[p];
        if (G < C) return MING_OK;  // too small to give every CTA work: stay on the per-kernel path
        std::vector<int> g0(C + 1);
        for (int i = 0; i <= C; i++) {
            // gate|up (p 2) is cut at whole tiles: each CTA finishes its SwiGLU features
            g0[i] = p == 2 ? (int)((long long)i * tiles[p] / C) * gpt[p] : (int)((long long)i * G / C);
        }
        int maxn = 0;
        for (int i = 0; i < C; i++) {
            maxn = std::max(maxn, g0[i + 1] - g0[i]);
        }
        if (p == 3 && maxn > MG_MAX_STAGE) return MING_OK;                // staged groups of h
        if ((maxn + MG_CWARPS - 1) / MG_CWARPS > gpt[p]) return MING_OK;  // a warp's run spans at most two tiles
        int* dg0 = c->mem.alloc<int>(C + 1, &rc);
        if (rc) return rc;
        CK(cudaMemcpy(dg0, g0.data(), (C + 1) * 4, cudaMemcpyHostToDevice));
        a.ph[p] = MegaPhase{dg0, nullptr, tiles[p], gpt[p]};
        if (p == 2) continue;  // gate|up: whole tiles per CTA
        // split-K phase: contributors per tile (the count every counted
        // accumulator word of the tile reaches when complete). Each consumer
        // warp of a CTA adds its own partial sums for the tiles its run of
        // the CTA's groups touches: warp w takes groups [w n / W, (w+1) n / W).
        if (tiles[p] > MG_MAX_TILES) return MING_OK;
        std::vector<int> tc(tiles[p], 0);
        for (int i = 0; i < C; i++) {
            const int n = g0[i + 1] - g0[i];
            for (int w = 0; w < MG_CWARPS; w++) {
                const int i0 = w * n / MG_CWARPS, i1 = (w + 1) * n / MG_CWARPS;
                if (i1 <= i0) continue;
                for (int t = (g0[i] + i0) / gpt[p]; t <= (g0[i] + i1 - 1) / gpt[p]; t++) tc[t]++;
            }
        }
        for (int t = 0; t < tiles[p]; t++)
            if (tc[t] < 1 || tc[t] > 255) return MING_OK;  // the count lives in one byte of the word
        int* dtc = c->mem.alloc<int>(tiles[p], &rc);
        if (rc) return rc;
        CK(cudaMemcpy(dtc, tc.data(), tiles[p] * 4, cudaMemcpyHostToDevice));
        a.ph[p].tcount = dtc;
    }
    if (nslots < 4) return MING_OK;  // warps consume a phase slot by slot: any ring works, a deeper one streams ahead
    if (f.max_ctx / PAGE + 1 > 512) return MING_OK;  // block-table rows live in shared memory
    // per-layer tables gathered into contiguous device arrays
    std::vector<const uint8_t*> wb((size_t)f.layers * MG_NPH);
    for (int l = 0; l < f.layers; l++) {
        wb[l * MG_NPH + 0] = c->layers[l].qkv.w.tiles;
        wb[l * MG_NPH + 1] = c->layers[l].o.w.tiles;
        wb[l * MG_NPH + 2] = c->layers[l].gu.w.tiles;
        wb[l * MG_NPH + 3] = c->layers[l].down.w.tiles;
    }
    const uint8_t** dwb = c->mem.alloc<const uint8_t*>(wb.size(), &rc);
    uint8_t* lpar = c->mem.alloc<uint8_t>((size_t)f.layers * lp_bytes, &rc);
    const int max_splits = (f.max_ctx + MG_ATT_CH - 1) / MG_ATT_CH;
    if (max_splits > 64) return MING_OK;  // a head's combine keeps up to 64 chunk maxima and sums in shared memory
    if (f.heads > 64) return MING_OK;      // the kernel's head -> kv head table has 64 entries
    if ((H / 64) * MG_MAXB * max_splits > 8192) return MING_OK;  // split weights live in the 32 KB fragment area
    const size_t attn_n = (size_t)MG_MAXB * f.heads * max_splits * MG_PART;
    uint64_t* attn = c->mem.alloc<uint64_t>(attn_n, &rc);
    const size_t comb_n = (size_t)MG_MAXB * f.heads * HD;
    uint64_t* comb = c->mem.alloc<uint64_t>(comb_n, &rc);
    const int acc_w = (std::max(qkv_rows, H) + 1) / 2 * 2;
    const size_t acc_n = (size_t)2 * f.layers * MG_NACC * MG_MAXB * acc_w;
    unsigned long long* acc = c->mem.alloc<unsigned long long>(acc_n, &rc);
    const size_t hbuf_n = (size_t)f.layers * MG_MAXB * f.ff;
    uint64_t* hbuf = c->mem.alloc<uint64_t>(hbuf_n, &rc);
    c->dev_err = c->mem.alloc<int>(1, &rc);
    c->mega_counter = c->mem.alloc<int>(2, &rc);
    if (rc) return rc;
    int* counter = c->mega_counter;
    c->mega_reset = [=]() -> cudaError_t {
        // a step that gave up leaves accumulators and tagged words of an
        // unfinished epoch: restart the epochs from zero on cleared buffers
        cudaError_t e = cudaMemset(acc, 0, acc_n * 8);
        if (e == cudaSuccess) e = cudaMemset(hbuf, 0, hbuf_n * 8);
        if (e == cudaSuccess) e = cudaMemset(attn, 0, attn_n * 8);
        if (e == cudaSuccess) e = cudaMemset(comb, 0, comb_n * 8);
        if (e == cudaSuccess) e = cudaMemset(counter, 0, 8);
        return e;
    };
    CK(c->mega_reset());
    CK(cudaMemcpy(dwb, wb.data(), wb.size() * sizeof(void*), cudaMemcpyHostToDevice));
    for (int l = 0; l < f.layers; l++) {
        uint8_t* blk = lpar + (size_t)l * lp_bytes;
        CK(cudaMemcpy(blk, c->layers[l].ln1, H * 2, cudaMemcpyDeviceToDevice));
        CK(cudaMemcpy(blk + 2 * H, c->layers[l].ln2, H * 2, cudaMemcpyDeviceToDevice));
        CK(cudaMemcpy(blk + 4 * H, c->layers[l].qkv.w.bias, qkv_rows * 4, cudaMemcpyDeviceToDevice));
    }
    a.wbase = dwb;
    a.lparams = lpar;
    a.lp_bytes = lp_bytes;
    a.norm = c->norm;
    a.stop_w = c->stop_w;
    a.stop_b = c->stop_b;
    a.kv = KvDev{c->pool, c->bt, c->bt_ld, f.layers, f.kv_heads};
    a.seq_len = c->seq_len;
    a.attn = attn;
    a.comb = comb;
    a.acc = acc;
    a.acc_w = acc_w;
    a.hbuf = hbuf;
    a.counter = c->mega_counter;
    a.err = c->dev_err;
    a.out_cell = c->out_cell;
    a.stop_cell = c->stop_cell;
    a.layers = f.layers;
    a.H = H;
    a.FF = f.ff;
    a.heads = f.heads;
    a.kvh = f.kv_heads;
    a.fmt = fmt;
    a.C = C;
    a.max_splits = max_splits;
    a.gps = gps;
    a.cb = cb;
    a.nslots = nslots;
    a.slot_bytes = slot;
    a.log2_theta = c->log2_theta;
    a.eps = f.rms_eps;
    const char* tr = getenv("MING_MEGA_TRACE");
    if (tr && std::string(tr) == "1") {
        // + 8 words: the CTAs' common-origin counter
        const size_t tn = (size_t)C * f.layers * MG_TRACE + 8;
        a.trace = c->mem.alloc<long long>(tn, &rc);
        if (rc) return rc;
        long long* sync = a.trace + (size_t)C * f.layers * MG_TRACE;
        c->mega_reset = [=, prev = c->mega_reset]() -> cudaError_t {
            cudaError_t e = prev();
            if (e == cudaSuccess) e = cudaMemset(sync, 0, 8);
            return e;
        };
    }
    c->mega_smem = mega_smem_bytes(nslots, slot, H, lp_bytes);
    c->mega_on = true;
    return MING_OK;
}

// Reads (and clears) the persistent kernel's device error flag.
int check_dev_err(ming_ctx* c) {
    if (!c->dev_err) return MING_OK;
    int e = 0;
    CK(cudaMemcpy(&e, c->dev_err, 4, cudaMemcpyDeviceToHost));
    if (e) {
        const int zero = 0;
        cudaMemcpy(c->dev_err, &zero, 4, cudaMemcpyHostToDevice);
        if (c->mega_reset) c->mega_reset();
        return fail(MING_ERR_CUDA, std::string(e == BK_ERR_WEIGHTS   ? "decode-batch linear: weight copy"
                                               : e == ATT_ERR_PAGES ? "attention: K/V page copy"
                                                                    : "persistent decode kernel") +
                                       ": a bounded device wait expired (code " + std::to_string(e) + ")");
    }
    return MING_OK;
}

int prepare_rows(ming_ctx* c, int B, const int* seq_ids, int steps) {
    if (B < 1 || B > c->cfg.max_batch) return fail(MING_ERR_INVALID, "batch size out of range");
    std::vector<int> ids(seq_ids, seq_ids + B);
    for (int i = 0; i < B; i++) {
        int rc = check_seq(c, ids[i]);
        if (rc) return rc;
        for (int j = 0; j < i; j++)
            if (ids[j] == ids[i]) return fail(MING_ERR_INVALID, "a sequence appears twice in one batch");
    }
    for (int i = 0; i < B; i++) {
        const int s = ids[i], len = c->seqs[s].len;
        if (len < 1) return fail(MING_ERR_INVALID, "decode needs a prefilled sequence");
        int rc = ensure_pages(c, s, len, len + steps);
        if (rc) return rc;
    }
    if ((int)c->row_seq_host.size() != B || !std::equal(ids.begin(), ids.end(), c->row_seq_host.begin())) {
        c->row_seq_host = ids;
        CK(cudaMemcpyAsync(c->row_seq, ids.data(), B * 4, cudaMemcpyHostToDevice, c->stream));
    }
    return MING_OK;
}

// ---- flow head ----

int cfm_token_enqueue(ming_ctx* c, int B, bool with_sde, float cfg, float shift, int step0, int nsteps) {
    const ming_cfg& f = c->cfg;
    const int H = f.dit_hidden, LAT = f.dit_latent, R = 6 * B;
    cudaStream_t s = c->stream;
    run_linear(c, c->c_emb.w, ProPlain{c->f_zc, f.dit_cond_dim, 0}, EpiAct{c->f_ce, nullptr, c->c_emb.w.bias, H, 0, H}, 2 * B,
               s);
    run_linear(c, c->x_emb.w, ProPlain{c->f_hist, LAT, 0}, EpiAct{c->f_xh, nullptr, c->x_emb.w.bias, H, 0, H}, B, s);
    for (int st = step0; st < step0 + nsteps; st++) {
        run_linear(c, c->x_emb.w, ProPlain{c->f_y, LAT, 0}, EpiAct{c->f_xy, nullptr, c->x_emb.w.bias, H, 0, H}, B, s);
        launch_tok_rows(c->temb + (size_t)st * H, c->f_ce, c->f_xh, c->f_xy, c->f_rows, B, H, s);
        for (auto& b : c->dit) {
            run_linear(c, b.qkv.w, ProRms{c->f_rows, b.norm1, H, H, 1e-6f, 0, nullptr},
                       EpiDitQKV{b.qkv.w.bias, c->f_qkv, c->inv_freq, H, 3, R}, R, s);
            launch_dit_attention(c->f_qkv, c->f_att, R, 3, H, f.dit_heads, s);
            run_linear(c, b.o.w, ProPlain{c->f_att, H, 0}, EpiResidual{c->f_rows, c->f_x1, b.o.w.bias, H}, R, s);
            run_linear(c, b.ff1.w, ProRms{c->f_x1, b.norm2, H, H, 1e-6f, 0, nullptr},
                       EpiAct{c->f_hh, nullptr, b.ff1.w.bias, f.dit_ff, 1, f.dit_ff}, R, s);
            run_linear(c, b.ff2.w, ProPlain{c->f_hh, f.dit_ff, 0}, EpiResidual{c->f_x1, c->f_rows, b.ff2.w.bias, H}, R, s);
        }
        launch_tok_final(c->f_rows, c->final_norm, c->final_w, c->final_b, c->f_y, with_sde ? c->f_sde : nullptr, st,
                         c->flow_dt[st], c->flow_sq[st], cfg, shift, B, H, LAT, s);
    }
    return MING_OK;
}

int cfm_ada_enqueue(ming_ctx* c, int B, bool with_sde, float cfg, float shift, int step0, int nsteps) {
    const ming_cfg& f = c->cfg;
    c->ktrace_used = 0;
    c->ktrace_used = 0;
    const int H = f.dit_hidden, LAT = f.dit_latent, F = f.dit_frames, NC = 2 * B, R = NC * F, MS = 6 * H;
    cudaStream_t s = c->stream;
    run_linear(c, c->c_emb.w, ProPlain{c->f_zc, f.dit_cond_dim, 0}, EpiAct{c->f_ce, nullptr, c->c_emb.w.bias, H, 0, H}, NC, s);
    // The modulations depend on the condition and the step's time embedding
    // only: SiLU(c + temb[st]) for every step of this call, then each block's
    // modulation linear (and the final layer's) over all of them at once — one
    // pass over each modulation weight per call instead of one per step.
    // Layout: block b's [nsteps][NC][6H] at f_mod + b * NR * 6H, the final
    // layer's [nsteps][NC][2H] after the blocks.
    const int NR = nsteps * NC;
    for (int k = 0; k < nsteps; k++)
        launch_ada_cond(c->temb + (size_t)(step0 + k) * H, c->f_ce, c->f_sc + (size_t)k * NC * H, NC, H, s);
    for (size_t bi = 0; bi < c->dit.size(); bi++) {
        auto& b = c->dit[bi];
        run_linear(c, b.ada.w, ProPlain{c->f_sc, H, 0}, EpiAct{c->f_mod + bi * NR * MS, nullptr, b.ada.w.bias, MS, 0, MS}, NR,
                   s);
    }
    uint16_t* fmod = c->f_mod + c->dit.size() * NR * MS;
    run_linear(c, c->final_ada.w, ProPlain{c->f_sc, H, 0}, EpiAct{fmod, nullptr, c->final_ada.w.bias, 2 * H, 0, 2 * H}, NR, s);
    for (int st = step0; st < step0 + nsteps; st++) {
        const size_t k = (size_t)(st - step0);
        run_linear(c, c->x_emb.w, ProLatent{c->f_y, B, F, LAT, 0}, EpiAct{c->f_rows, nullptr, c->x_emb.w.bias, H, 0, H}, R, s);
        for (size_t bi = 0; bi < c->dit.size(); bi++) {
            auto& b = c->dit[bi];
            const uint16_t* mod = c->f_mod + bi * NR * MS + k * NC * MS;
            run_linear(c, b.qkv.w, ProLnMod{c->f_rows, mod, mod + H, H, MS, H, F, 0, nullptr},
                       EpiDitQKV{b.qkv.w.bias, c->f_qkv, c->inv_freq, H, F, R}, R, s);
            launch_dit_attention(c->f_qkv, c->f_att, R, F, H, f.dit_heads, s);
            run_linear(c, b.o.w, ProPlain{c->f_att, H, 0}, EpiGatedRes{c->f_rows, c->f_rows, b.o.w.bias, mod + 2 * H, H, MS, F},
                       R, s);
            run_linear(c, b.ff1.w, ProLnMod{c->f_rows, mod + 3 * H, mod + 4 * H, H, MS, H, F, 0, nullptr},
                       EpiAct{c->f_hh, nullptr, b.ff1.w.bias, f.dit_ff, 1, f.dit_ff}, R, s);
            run_linear(c, b.ff2.w, ProPlain{c->f_hh, f.dit_ff, 0},
                       EpiGatedRes{c->f_rows, c->f_rows, b.ff2.w.bias, mod + 5 * H, H, MS, F}, R, s);
        }
        const uint16_t* fm = fmod + k * NC * 2 * H;
        run_linear(c, c->final_lin.w, ProLnMod{c->f_rows, fm, fm + H, H, 2 * H, H, F, 0, nullptr},
                   EpiAct{nullptr, c->f_vel, c->final_lin.w.bias, LAT, 3, LAT}, R, s);
        launch_ada_euler(c->f_vel, c->f_y, with_sde ? c->f_sde : nullptr, st, c->flow_dt[st], c->flow_sq[st], cfg, shift, B,
                         F, LAT, s);
    }
    return MING_OK;
}

int cfm_enqueue(ming_ctx* c, int B, bool with_sde, float cfg, float shift, int step0, int nsteps) {
    if (c->cfg.dit_mode == MING_DIT_ADALN) return cfm_ada_enqueue(c, B, with_sde, cfg, shift, step0, nsteps);
    return cfm_token_enqueue(c, B, with_sde, cfg, shift, step0, nsteps);
}

int agg_enqueue(ming_ctx* c, int B, const uint16_t* latent) {
    const ming_cfg& f = c->cfg;
    cudaStream_t s = c->stream;
    if (c->agg_proj_on) {
        // adaLN head: latent [B][dit_frames][dit_latent] -> [B][hidden]
        launch_latent_mean(latent, c->a_mean, B, f.dit_frames, f.dit_latent, s);
        run_linear(c, c->agg_proj.w, ProPlain{c->a_mean, f.dit_latent, 0},
                   EpiAct{c->a_out, nullptr, c->agg_proj.w.bias, f.hidden, 0, f.hidden}, B, s);
        return MING_OK;
    }
    if (c->agg.empty()) return fail(MING_ERR_INVALID, "no aggregator configured");
    const int H = f.dit_hidden, R = 2 * B;
    run_linear(c, c->agg_x_emb.w, ProPlain{latent, f.dit_latent, 0}, EpiAct{c->a_xe, nullptr, c->agg_x_emb.w.bias, H, 0, H}, B,
               s);
    // rows [cls, x_emb(latent)] per sequence
    for (int b = 0; b < B; b++)
        CK(cudaMemcpyAsync(c->a_rows + (size_t)(2 * b) * H, c->agg_cls, (size_t)H * 2, cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpy2DAsync(c->a_rows + H, (size_t)2 * H * 2, c->a_xe, (size_t)H * 2, (size_t)H * 2, B, cudaMemcpyDeviceToDevice,
                         s));
    for (auto& b : c->agg) {
        run_linear(c, b.qkv.w, ProRms{c->a_rows, b.norm1, H, H, 1e-6f, 0, nullptr},
                   EpiDitQKV{b.qkv.w.bias, c->a_qkv, c->agg_inv_freq, H, 2, R}, R, s);
        launch_dit_attention(c->a_qkv, c->a_att, R, 2, H, f.dit_heads, s);
        run_linear(c, b.o.w, ProPlain{c->a_att, H, 0}, EpiResidual{c->a_rows, c->a_x1, b.o.w.bias, H}, R, s);
        run_linear(c, b.ff1.w, ProRms{c->a_x1, b.norm2, H, H, 1e-6f, 0, nullptr},
                   EpiAct{c->a_hh, nullptr, b.ff1.w.bias, f.dit_ff, 1, f.dit_ff}, R, s);
        run_linear(c, b.ff2.w, ProPlain{c->a_hh, f.dit_ff, 0}, EpiResidual{c->a_x1, c->a_rows, b.ff2.w.bias, H}, R, s);
    }
    // final RMSNorm + linear on each CLS row (row stride 2H selects them)
    run_linear(c, c->agg_final.w, ProRmsGraph{c->a_rows, c->agg_norm, 2 * H, H, 1e-6f, 0, nullptr},
               EpiAct{c->a_out, nullptr, c->agg_final.w.bias, f.hidden, 0, f.hidden}, B, s);
    return MING_OK;
}

int seq_release(ming_ctx* c, int id) {
    int rc = check_seq(c, id);
    if (rc) return rc;
    for (int p = 0; p < c->bt_ld; p++) {
        int& e = c->bt_host[(size_t)id * c->bt_ld + p];
        if (e >= 0) c->free_pages.push_back(e);
        e = -1;
    }
    // -1 bytes are 0xff: the whole row reset in one queued fill
    CK(cudaMemsetAsync(c->bt + (size_t)id * c->bt_ld, 0xff, (size_t)c->bt_ld * 4, c->stream));
    c->seqs[id] = SeqInfo{};
    return MING_OK;
}

}  // namespace rt
}  // namespace ming

// ---------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------

extern "C" {

const char* ming_cuda_last_error(void) { return g_err.c_str(); }

void ming_cuda_default_cfg(ming_cfg* c) {
    std::memset(c, 0, sizeof(*c));
    c->hidden = 896;
    c->layers = 24;
    c->heads = 14;
    c->kv_heads = 2;
    c->head_dim = 64;
    c->ff = 4864;
    c->rope_theta = 1e6f;
    c->rms_eps = 1e-6f;
    c->weight_bits = 16;
    c->group_size = 64;
    c->page_size = 16;
    c->max_seqs = 64;
    c->max_ctx = 4096;
    c->max_pages = 4096;
    c->max_batch = 64;
    c->max_prefill = 256;
    c->dit_mode = MING_DIT_TOKEN;
    c->dit_hidden = 1024;
    c->dit_blocks = 8;
    c->dit_heads = 16;
    c->dit_ff = 4096;
    c->dit_latent = 64;
    c->dit_frames = 1;
    c->dit_cond_dim = 896;
    c->dit_freq_dim = 256;
    c->dit_max_batch = 32;
    c->agg_blocks = 8;
    c->vae_layers = 0;
    c->vae_ff = 4864;
    c->vae_window = 64;
    c->vae_max_latents = 512;
}

int ming_cuda_create(int device, const ming_cfg* cfg, ming_ctx** out) {
    if (!cfg || !out) return fail(MING_ERR_INVALID, "null argument");
    const ming_cfg& f = *cfg;
    if (f.head_dim != 64) return fail(MING_ERR_INVALID, "head_dim must be 64");
    if (f.page_size != PAGE) return fail(MING_ERR_INVALID, "page_size must be 16");
    if (f.hidden % 64 || f.ff % 64 || f.hidden != f.heads * 64)
        return fail(MING_ERR_INVALID, "hidden and ff must be multiples of 64, hidden = heads*64");
    if (f.kv_heads < 1 || f.heads % f.kv_heads || f.heads / f.kv_heads > 8)
        return fail(MING_ERR_INVALID, "heads must be a multiple of kv_heads with at most 8 per group");
    if (f.group_size != 64) return fail(MING_ERR_INVALID, "group_size must be 64");
    if (f.max_ctx < PAGE || f.max_ctx % ATT_SPLIT) return fail(MING_ERR_INVALID, "max_ctx must be a multiple of 256");
    if (f.max_batch < 1 || f.max_batch > 256 || f.max_prefill < 1 || f.max_seqs < 1 || f.max_pages < 1)
        return fail(MING_ERR_INVALID, "bad batch/prefill/sequence/page limits");
    if (f.dit_mode != MING_DIT_NONE) {
        if (f.dit_hidden % 64 || f.dit_ff % 64 || f.dit_hidden != f.dit_heads * 64 || f.dit_latent % 16 ||
            f.dit_cond_dim % 64 || f.dit_freq_dim % 64 || f.dit_max_batch < 1)
            return fail(MING_ERR_INVALID, "bad flow-head shape");
        if (f.dit_mode == MING_DIT_TOKEN && f.dit_frames != 1) return fail(MING_ERR_INVALID, "token mode has one frame");
        if (f.dit_mode == MING_DIT_ADALN && (f.dit_frames < 1 || f.dit_frames > 16))
            return fail(MING_ERR_INVALID, "adaLN frames must be 1..16");
    }
    int ndev = 0;
    CK(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(MING_ERR_INVALID, "no such CUDA device");
    CK(cudaSetDevice(device));
    std::unique_ptr<ming_ctx> c(new ming_ctx());
    c->device = device;
    c->cfg = f;
    CK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
    *out = c.release();
    return MING_OK;
}

int ming_cuda_load_tensor(ming_ctx* c, const char* name, int dtype, const int64_t* shape, int ndim, const void* host) {
    if (!c || !name || (!shape && ndim) || !host || ndim < 0 || ndim > 4) return fail(MING_ERR_INVALID, "bad argument");
    if (c->finalized) return fail(MING_ERR_INVALID, "context already finalized");
    if (dtype != MING_DTYPE_BF16 && dtype != MING_DTYPE_F32 && dtype != MING_DTYPE_U32)
        return fail(MING_ERR_INVALID, "unsupported dtype");
    HostTensor t;
    t.dtype = dtype;
    int64_t n = 1;
    for (int i = 0; i < ndim; i++) {
        if (shape[i] < 0) return fail(MING_ERR_INVALID, "negative dimension");
        t.shape.push_back(shape[i]);
        n *= shape[i];
    }
    const size_t bytes = (size_t)n * (dtype == MING_DTYPE_BF16 ? 2 : 4);
    t.data.resize(bytes);
    std::memcpy(t.data.data(), host, bytes);
    c->staged[name] = std::move(t);
    return MING_OK;
}

int ming_cuda_finalize(ming_ctx* c) {
    if (!c) return fail(MING_ERR_INVALID, "null context");
    if (c->finalized) return MING_OK;
    CK(cudaSetDevice(c->device));
    const ming_cfg& f = c->cfg;
    int rc;
    // ---- LM (layers == 0: a flow-head-only context) ----
    c->layers.resize(f.layers);
    const int H = f.hidden, QD = f.heads * 64, KD = f.kv_heads * 64;
    for (int l = 0; l < f.layers; l++) {
        const std::string p = "model.model.layers." + std::to_string(l);
        auto& L = c->layers[l];
        LinearSrc q, k, v, o, g, u, d;
        if ((rc = lin_src(c, p + ".self_attn.q_proj", q, true))) return rc;
        if ((rc = lin_src(c, p + ".self_attn.k_proj", k, true))) return rc;
        if ((rc = lin_src(c, p + ".self_attn.v_proj", v, true))) return rc;
        if ((rc = lin_src(c, p + ".self_attn.o_proj", o, false))) return rc;
        if ((rc = lin_src(c, p + ".mlp.gate_proj", g, false))) return rc;
        if ((rc = lin_src(c, p + ".mlp.up_proj", u, false))) return rc;
        if ((rc = lin_src(c, p + ".mlp.down_proj", d, false))) return rc;
        if (q.out != QD || k.out != KD || v.out != KD || q.in != H || o.out != H || o.in != QD || g.out != f.ff ||
            u.out != f.ff || d.out != H || d.in != f.ff)
            return fail(MING_ERR_INVALID, p + ": linear shapes do not match the config");
        if (q.fmt != f.weight_bits || o.fmt != f.weight_bits || g.fmt != f.weight_bits || d.fmt != f.weight_bits)
            return fail(MING_ERR_INVALID, p + ": weight format differs from cfg.weight_bits");
        // q|k|v: tile t of a block covers head t/4, dims d0 = 8(t%4)..+7 and d0+32..+39
        std::vector<RowRef> rows;
        const int nh[3] = {f.heads, f.kv_heads, f.kv_heads};
        for (int b = 0; b < 3; b++)
            for (int t = 0; t < nh[b] * 4; t++)
                for (int r = 0; r < 16; r++) {
                    const int h = t / 4, d0 = (t % 4) * 8;
                    rows.push_back({b, h * 64 + (r < 8 ? d0 + r : 32 + d0 + r - 8)});
                }
        if ((rc = upload_packed(c, {q, k, v},
                                {p + ".self_attn.q_proj.weight", p + ".self_attn.k_proj.weight", p + ".self_attn.v_proj.weight"},
                                rows, L.qkv)))
            return rc;
        rows.clear();
        for (int i = 0; i < H; i++) rows.push_back({0, i});
        if ((rc = upload_packed(c, {o}, {p + ".self_attn.o_proj.weight"}, rows, L.o))) return rc;
        if ((rc = upload_packed(c, {d}, {p + ".mlp.down_proj.weight"}, rows, L.down))) return rc;
        rows.clear();
        for (int t = 0; t < f.ff / 8; t++)
            for (int r = 0; r < 16; r++) rows.push_back({r < 8 ? 0 : 1, t * 8 + (r & 7)});
        if ((rc = upload_packed(c, {g, u}, {p + ".mlp.gate_proj.weight", p + ".mlp.up_proj.weight"}, rows, L.gu))) return rc;
        L.ln1_unit = unit_gains(c, p + ".input_layernorm.weight");
        L.ln2_unit = unit_gains(c, p + ".post_attention_layernorm.weight");
        if ((rc = upload_raw(c, p + ".input_layernorm.weight", MING_DTYPE_BF16, H, (void**)&L.ln1))) return rc;
        if ((rc = upload_raw(c, p + ".post_attention_layernorm.weight", MING_DTYPE_BF16, H, (void**)&L.ln2))) return rc;
    }
    if (f.layers > 0) {
        if ((rc = upload_raw(c, "model.model.norm.weight", MING_DTYPE_BF16, H, (void**)&c->norm))) return rc;
        if ((rc = upload_raw(c, "stop_head.weight", MING_DTYPE_BF16, 2 * H, (void**)&c->stop_w))) return rc;
        if ((rc = upload_raw(c, "stop_head.bias", MING_DTYPE_BF16, 2, (void**)&c->stop_b))) return rc;
    }
    c->log2_theta = log2f(f.rope_theta);

    // ---- KV pool, step state, activations ----
    c->bt_ld = f.max_ctx / PAGE;
    c->nsplit = f.max_ctx / ATT_SPLIT;
    c->maxr = std::max(f.max_batch, f.max_prefill);
    const size_t page_elems = (size_t)f.layers * 2 * f.kv_heads * PAGE * 64;
    rc = MING_OK;
    c->pool = c->mem.alloc<uint16_t>((size_t)f.max_pages * page_elems, &rc);
    c->bt = c->mem.alloc<int>((size_t)f.max_seqs * c->bt_ld, &rc);
    c->x = c->mem.alloc<uint16_t>((size_t)c->maxr * H, &rc);
    c->x1 = c->mem.alloc<uint16_t>((size_t)c->maxr * H, &rc);
    c->q = c->mem.alloc<uint16_t>((size_t)c->maxr * QD, &rc);
    c->att = c->mem.alloc<uint16_t>((size_t)c->maxr * f.heads * HD, &rc);
    c->h = c->mem.alloc<uint16_t>((size_t)c->maxr * f.ff, &rc);
    c->z = c->mem.alloc<uint16_t>((size_t)c->maxr * H, &rc);
    c->stop = c->mem.alloc<float>(c->maxr, &rc);
    c->part = c->mem.alloc<float>((size_t)c->maxr * c->nsplit * f.heads * PART_STRIDE, &rc);
    c->seq_len = c->mem.alloc<int>(f.max_seqs, &rc);
    c->row_seq = c->mem.alloc<int>(c->maxr, &rc);
    c->row_pos = c->mem.alloc<int>(c->maxr, &rc);
    c->step_counter = c->mem.alloc<int>(2, &rc);
    c->out_cell = c->mem.alloc<uint16_t*>(1, &rc);
    c->stop_cell = c->mem.alloc<float*>(1, &rc);
    if (rc) return rc;
    if ((long long)f.max_pages * f.layers * 2 * f.kv_heads * PAGE >= (1LL << 31))
        return fail(MING_ERR_INVALID, "max_pages x layers x 2 x kv_heads x 16 must stay below 2^31 (the page copies' row coordinate)");
    if (f.layers > 0 && !make_kv_tensor_map(&c->kv_tmap, c->pool, (long long)f.max_pages * f.layers * 2 * f.kv_heads * PAGE))
        return fail(MING_ERR_CUDA, "the KV page pool's tensor map could not be encoded (cuTensorMapEncodeTiled)");
    c->bt_host.assign((size_t)f.max_seqs * c->bt_ld, -1);
    CK(cudaMemcpy(c->bt, c->bt_host.data(), c->bt_host.size() * 4, cudaMemcpyHostToDevice));
    for (int p = f.max_pages - 1; p >= 0; p--) c->free_pages.push_back(p);
    c->seqs.assign(f.max_seqs, SeqInfo{});
    if (f.layers > 0 && (rc = setup_mega(c))) return rc;

    // ---- flow head ----
    if (f.dit_mode != MING_DIT_NONE) {
        const int DH = f.dit_hidden, LAT = f.dit_latent, MB = f.dit_max_batch;
        const bool ada = f.dit_mode == MING_DIT_ADALN;
        const std::string F = ada ? "adaln_head" : "flowloss.cfm.model";
        if ((rc = load_dit_blocks(c, F, f.dit_blocks, DH, ada, c->dit))) return rc;
        if ((rc = pack_plain(c, F + ".t_embedder.time_mlp.0", true, c->t_mlp0))) return rc;
        if ((rc = pack_plain(c, F + ".t_embedder.time_mlp.2", true, c->t_mlp2))) return rc;
        if ((rc = pack_plain(c, F + ".x_embedder", true, c->x_emb))) return rc;
        if ((rc = pack_plain(c, F + ".c_embedder.cond_embedder", true, c->c_emb))) return rc;
        if ((rc = upload_raw(c, F + ".rotary_embed.inv_freq", MING_DTYPE_F32, 32, (void**)&c->inv_freq))) return rc;
        if (ada) {
            if ((rc = pack_plain(c, F + ".final_layer.adaLN_modulation.1", true, c->final_ada))) return rc;
            if ((rc = pack_plain(c, F + ".final_layer.linear", true, c->final_lin))) return rc;
        } else {
            if ((rc = upload_raw(c, F + ".final_layer.norm_final.weight", MING_DTYPE_BF16, DH, (void**)&c->final_norm))) return rc;
            if ((rc = upload_raw(c, F + ".final_layer.linear.weight", MING_DTYPE_BF16, (int64_t)LAT * DH, (void**)&c->final_w)))
                return rc;
            if ((rc = upload_raw(c, F + ".final_layer.linear.bias", MING_DTYPE_BF16, LAT, (void**)&c->final_b))) return rc;
        }
        if (c->c_emb.w.K != f.dit_cond_dim || c->x_emb.w.K != LAT || c->t_mlp0.w.K != f.dit_freq_dim)
            return fail(MING_ERR_INVALID, "flow head input dims do not match the config");
        const int F_ = f.dit_frames, rows = ada ? 2 * MB * F_ : 6 * MB;
        rc = MING_OK;
        c->f_zc = c->mem.alloc<uint16_t>((size_t)2 * MB * f.dit_cond_dim, &rc);
        c->f_hist = c->mem.alloc<uint16_t>((size_t)MB * LAT, &rc);
        c->f_y = c->mem.alloc<uint16_t>((size_t)MB * F_ * LAT, &rc);
        c->f_sde = c->mem.alloc<uint16_t>((size_t)10 * MB * F_ * LAT, &rc);
        c->f_ce = c->mem.alloc<uint16_t>((size_t)2 * MB * DH, &rc);
        c->f_xh = c->mem.alloc<uint16_t>((size_t)MB * DH, &rc);
        c->f_xy = c->mem.alloc<uint16_t>((size_t)MB * DH, &rc);
        c->f_rows = c->mem.alloc<uint16_t>((size_t)rows * DH, &rc);
        c->f_x1 = c->mem.alloc<uint16_t>((size_t)rows * DH, &rc);
        c->f_qkv = c->mem.alloc<uint16_t>((size_t)3 * rows * DH, &rc);
        c->f_att = c->mem.alloc<uint16_t>((size_t)rows * DH, &rc);
        c->f_hh = c->mem.alloc<uint16_t>((size_t)rows * f.dit_ff, &rc);
        // adaLN: every step's SiLU(c + temb) and modulations of one call (up to 10 steps)
        const size_t nsc = f.dit_mode == MING_DIT_ADALN ? 10 : 1;
        c->f_sc = c->mem.alloc<uint16_t>(nsc * 2 * MB * DH, &rc);
        c->f_mod = c->mem.alloc<uint16_t>(nsc * 2 * MB * ((size_t)f.dit_blocks * 6 * DH + 2 * DH), &rc);
        c->f_vel = c->mem.alloc<float>((size_t)rows * LAT, &rc);
        if (rc) return rc;
        if ((rc = build_temb(c, f.dit_freq_dim, DH))) return rc;
    }
    // ---- aggregator ----
    if (f.agg_blocks > 0 && f.dit_mode == MING_DIT_TOKEN) {
        const int DH = f.dit_hidden, MB = f.dit_max_batch;
        const std::string A = "linear_proj_audio";
        if ((rc = load_dit_blocks(c, A, f.agg_blocks, DH, false, c->agg))) return rc;
        if ((rc = pack_plain(c, A + ".x_embedder", true, c->agg_x_emb))) return rc;
        if ((rc = pack_plain(c, A + ".final_layer.linear", true, c->agg_final))) return rc;
        if ((rc = upload_raw(c, A + ".word_embedder.weight", MING_DTYPE_BF16, DH, (void**)&c->agg_cls))) return rc;
        if ((rc = upload_raw(c, A + ".final_layer.norm_final.weight", MING_DTYPE_BF16, DH, (void**)&c->agg_norm))) return rc;
        if ((rc = upload_raw(c, A + ".rotary_embed.inv_freq", MING_DTYPE_F32, 32, (void**)&c->agg_inv_freq))) return rc;
        rc = MING_OK;
        c->a_lat = c->mem.alloc<uint16_t>((size_t)MB * f.dit_latent, &rc);
        c->a_xe = c->mem.alloc<uint16_t>((size_t)MB * DH, &rc);
        c->a_rows = c->mem.alloc<uint16_t>((size_t)2 * MB * DH, &rc);
        c->a_x1 = c->mem.alloc<uint16_t>((size_t)2 * MB * DH, &rc);
        c->a_qkv = c->mem.alloc<uint16_t>((size_t)6 * MB * DH, &rc);
        c->a_att = c->mem.alloc<uint16_t>((size_t)2 * MB * DH, &rc);
        c->a_hh = c->mem.alloc<uint16_t>((size_t)2 * MB * f.dit_ff, &rc);
        c->a_out = c->mem.alloc<uint16_t>((size_t)MB * f.hidden, &rc);
        if (rc) return rc;
    }
    // ---- adaLN head: the latent's path into the next LM input, when the
    //      checkpoint has it (mean of the patch's frames, then a linear
    //      latent -> hidden; no reference code, the choice is pinned here) ----
    if (f.dit_mode == MING_DIT_ADALN && c->staged.count("aggregator.proj.weight")) {
        const int MB = f.dit_max_batch;
        int od = 0;
        if ((rc = pack_plain(c, "aggregator.proj", true, c->agg_proj, &od))) return rc;
        if (c->agg_proj.w.K != f.dit_latent || od != f.hidden)
            return fail(MING_ERR_INVALID, "aggregator.proj must be [hidden, dit_latent]");
        rc = MING_OK;
        c->a_lat = c->mem.alloc<uint16_t>((size_t)MB * f.dit_frames * f.dit_latent, &rc);
        c->a_mean = c->mem.alloc<uint16_t>((size_t)MB * f.dit_latent, &rc);
        c->a_out = c->mem.alloc<uint16_t>((size_t)MB * f.hidden, &rc);
        if (rc) return rc;
        c->agg_proj_on = true;
    }
    if (f.vae_layers > 0 && (rc = vae_finalize(c))) return rc;
    {
        // staging scratch of the many-row linears: every (rows, K) a linear of
        // this context can see; larger calls fall back to in-kernel staging
        int rows_cap = c->maxr, k_cap = std::max(std::max(f.hidden, f.ff), f.heads * HD);
        if (f.vae_layers > 0) {
            // the decoder's rows (4 per latent) and its doubled / tripled K
            rows_cap = std::max(rows_cap, 4 * f.vae_max_latents);
            k_cap = std::max(k_cap, std::max(2 * std::max(f.hidden, f.vae_ff), (int)c->vae_dft.w.K));
        }
        if (f.dit_mode != MING_DIT_NONE) {
            const int MB = f.dit_max_batch;
            rows_cap = std::max(rows_cap, std::max(2 * MB * f.dit_frames, 20 * MB));  // 20 MB: 10 steps' modulation rows
            k_cap = std::max(k_cap, std::max(std::max(f.dit_hidden, f.dit_ff), std::max(f.dit_cond_dim, f.dit_freq_dim)));
        }
        if (f.weight_bits != 16 && f.max_prefill > 64 && tc_copies_enabled())
            k_cap = std::max(k_cap, 2 * std::max(f.hidden, f.ff));  // the prefill copies' rows, staged twice
        rows_cap = (rows_cap + 255) / 256 * 256;  // the tcgen05 linear reads whole 256-row blocks
        k_cap = (k_cap + 63) / 64 * 64;
        rc = MING_OK;
        c->lin.frag = c->mem.alloc<uint2>((size_t)rows_cap / 8 * (k_cap / 16) * 32, &rc);
        c->lin.ysum = c->mem.alloc<float>((size_t)rows_cap / 8 * (k_cap / 64) * 8, &rc);
        c->lin.post = c->mem.alloc<float>(rows_cap, &rc);
        if (rc) return rc;
        c->lin.rows = rows_cap;
        c->lin.K = k_cap;
        CK(cudaDeviceGetAttribute(&c->lin.sms, cudaDevAttrMultiProcessorCount, c->device));
        if (!c->dev_err) c->dev_err = c->mem.alloc<int>(1, &rc);
        if (rc) return rc;
        if (!c->err_host && cudaHostAlloc(reinterpret_cast<void**>(&c->err_host), 4, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            c->err_host = nullptr;  // the error flag is then read with a synchronous copy
        }
        c->lin.err = c->dev_err;
        const char* kt = getenv("MING_KTRACE");
        if (kt && std::string(kt) == "1") {
            c->ktrace = c->mem.alloc<long long>((size_t)KT_SLOTS * KT_CTAS * 8, &rc);
            if (rc) return rc;
        }
    }
    CK(cudaDeviceSynchronize());
    c->staged.clear();
    c->finalized = true;
    return MING_OK;
}

int ming_cuda_seq_alloc(ming_ctx* c, int* id) {
    if (!c || !id || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    for (int i = 0; i < (int)c->seqs.size(); i++)
        if (!c->seqs[i].live) {
            c->seqs[i] = SeqInfo{true, 0};
            const int zero = 0;
            CK(cudaMemcpyAsync(c->seq_len + i, &zero, 4, cudaMemcpyHostToDevice, c->stream));
            *id = i;
            return MING_OK;
        }
    return fail(MING_ERR_NOMEM, "all sequence slots are in use");
}

int ming_cuda_seq_free(ming_ctx* c, int id) {
    if (!c) return fail(MING_ERR_INVALID, "null context");
    int rc = check_seq(c, id);
    if (rc) return rc;
    if ((rc = seq_release(c, id))) return rc;
    CK(cudaStreamSynchronize(c->stream));
    return MING_OK;
}

int ming_cuda_seq_len(ming_ctx* c, int id, int* len) {
    if (!c || !len) return fail(MING_ERR_INVALID, "null argument");
    int rc = check_seq(c, id);
    if (rc) return rc;
    *len = c->seqs[id].len;
    return MING_OK;
}

int ming_cuda_seq_truncate(ming_ctx* c, int id, int len) {
    if (!c) return fail(MING_ERR_INVALID, "null context");
    int rc = check_seq(c, id);
    if (rc) return rc;
    if (len < 0 || len > c->seqs[id].len) return fail(MING_ERR_INVALID, "truncate length out of range");
    c->seqs[id].len = len;
    CK(cudaMemcpyAsync(c->seq_len + id, &c->seqs[id].len, 4, cudaMemcpyHostToDevice, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return MING_OK;
}

int ming_cuda_lm_prefill(ming_ctx* c, int s, const uint16_t* x, int L, uint16_t* out, float* stop, int kind) {
    if (!c || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    if (c->cfg.layers < 1) return fail(MING_ERR_INVALID, "no LM configured");
    if (!x || L < 1) return fail(MING_ERR_INVALID, "empty prompt");
    int rc = check_seq(c, s);
    if (rc) return rc;
    CK(cudaSetDevice(c->device));
    const int H = c->cfg.hidden, start = c->seqs[s].len;
    if ((rc = ensure_pages(c, s, start, start + L))) return rc;
    c->row_seq_host.clear();  // row_seq is overwritten below
    std::vector<int> seqv(c->cfg.max_prefill, s), posv(c->cfg.max_prefill);
    for (int c0 = 0; c0 < L; c0 += c->cfg.max_prefill) {
        const int n = std::min(c->cfg.max_prefill, L - c0);
        for (int r = 0; r < n; r++) posv[r] = start + c0 + r;
        CK(cudaMemcpyAsync(c->row_seq, seqv.data(), n * 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(c->row_pos, posv.data(), n * 4, cudaMemcpyHostToDevice, c->stream));
        if ((rc = copy_in(c, c->x, x + (size_t)c0 * H, (size_t)n * H * 2, kind))) return rc;
        const cudaError_t le = enqueue_layers(c, n, false);
        if (le != cudaSuccess) return fail(MING_ERR_CUDA, std::string("prefill attention launch: ") + cudaGetErrorString(le));
        if (out || stop) {
            launch_final(FinalArgs{c->x, c->norm, c->stop_w, c->stop_b, c->z, c->stop, nullptr, step_dev(c), H, 0, 0,
                                   c->cfg.rms_eps},
                         n, c->stream);
            if ((rc = copy_out(c, out ? out + (size_t)c0 * H : nullptr, c->z, (size_t)n * H * 2, kind))) return rc;
            if ((rc = copy_out(c, stop ? stop + c0 : nullptr, c->stop, (size_t)n * 4, kind))) return rc;
        }
        if (kind == MING_PTR_HOST) CK(cudaStreamSynchronize(c->stream));
    }
    CK(cudaGetLastError());
    c->seqs[s].len = start + L;
    CK(cudaMemcpyAsync(c->seq_len + s, &c->seqs[s].len, 4, cudaMemcpyHostToDevice, c->stream));
    if (kind == MING_PTR_HOST) CK(cudaStreamSynchronize(c->stream));
    return MING_OK;
}

int ming_cuda_lm_decode(ming_ctx* c, int B, const int* ids, const uint16_t* x, uint16_t* out, float* stop, int kind) {
    if (!c || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    if (c->cfg.layers < 1) return fail(MING_ERR_INVALID, "no LM configured");
    if (!ids || !x) return fail(MING_ERR_INVALID, "null argument");
    CK(cudaSetDevice(c->device));
    int rc = prepare_rows(c, B, ids, 1);
    if (rc) return rc;
    const int H = c->cfg.hidden;
    cudaGraphExec_t g;
    if ((rc = decode_graph(c, B, &g))) return rc;
    if (!c->cells_null) {
        // the step's kernels write per-step outputs only through non-null
        // cells (generate); the cells stay null until the next generate
        static uint16_t* const null_out = nullptr;
        static float* const null_stop = nullptr;
        CK(cudaMemcpyAsync(c->out_cell, &null_out, sizeof(void*), cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(c->stop_cell, &null_stop, sizeof(void*), cudaMemcpyHostToDevice, c->stream));
        c->cells_null = true;
    }
    if ((rc = copy_in(c, c->x, x, (size_t)B * H * 2, kind))) return rc;
    CK(cudaGraphLaunch(g, c->stream));
    for (int i = 0; i < B; i++) c->seqs[ids[i]].len += 1;
    if ((rc = copy_out(c, out, c->z, (size_t)B * H * 2, kind))) return rc;
    if ((rc = copy_out(c, stop, c->stop, (size_t)B * 4, kind))) return rc;
    if (kind == MING_PTR_HOST) {
        if (c->err_host && c->dev_err) {
            // the error flag travels with the outputs: one synchronisation
            CK(cudaMemcpyAsync(c->err_host, c->dev_err, 4, cudaMemcpyDeviceToHost, c->stream));
            CK(cudaStreamSynchronize(c->stream));
            if (*c->err_host) return check_dev_err(c);
        } else {
            CK(cudaStreamSynchronize(c->stream));
            if ((rc = check_dev_err(c))) return rc;
        }
    }
    return MING_OK;
}

int ming_cuda_lm_generate(ming_ctx* c, int B, const int* ids, const uint16_t* x0, int steps, uint16_t* out, float* stop,
                          int kind) {
    if (!c || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    if (c->cfg.layers < 1) return fail(MING_ERR_INVALID, "no LM configured");
    if (!ids || !x0 || steps < 1) return fail(MING_ERR_INVALID, "bad argument");
    CK(cudaSetDevice(c->device));
    int rc = prepare_rows(c, B, ids, steps);
    if (rc) return rc;
    const int H = c->cfg.hidden;
    cudaGraphExec_t g;
    if ((rc = decode_graph(c, B, &g))) return rc;
    uint16_t* o = nullptr;
    float* sp = nullptr;
    if (out) {
        if (kind == MING_PTR_DEVICE) o = out;
        else {
            const size_t need = (size_t)steps * B * H;
            if (c->gen_out_elems < need) {
                if (c->gen_out) cudaFree(c->gen_out);
                c->gen_out = nullptr;
                c->gen_out_elems = 0;
                CK(cudaMalloc(&c->gen_out, need * 2));
                c->gen_out_elems = need;
            }
            o = c->gen_out;
        }
    }
    if (stop) {
        if (kind == MING_PTR_DEVICE) sp = stop;
        else {
            const size_t need = (size_t)steps * B;
            if (c->gen_stop_elems < need) {
                if (c->gen_stop) cudaFree(c->gen_stop);
                c->gen_stop = nullptr;
                c->gen_stop_elems = 0;
                CK(cudaMalloc(&c->gen_stop, need * 4));
                c->gen_stop_elems = need;
            }
            sp = c->gen_stop;
        }
    }
    CK(cudaMemcpyAsync(c->out_cell, &o, sizeof(void*), cudaMemcpyHostToDevice, c->stream));
    CK(cudaMemcpyAsync(c->stop_cell, &sp, sizeof(void*), cudaMemcpyHostToDevice, c->stream));
    c->cells_null = !o && !sp;
    CK(cudaMemsetAsync(c->step_counter, 0, 8, c->stream));
    if (c->mega_counter) CK(cudaMemsetAsync(c->mega_counter + 1, 0, 4, c->stream));  // the epoch is never reset
    if ((rc = copy_in(c, c->x, x0, (size_t)B * H * 2, kind))) return rc;
    for (int i = 0; i < steps; i++) CK(cudaGraphLaunch(g, c->stream));
    for (int i = 0; i < B; i++) c->seqs[ids[i]].len += steps;
    if (kind == MING_PTR_HOST) {
        if (out) CK(cudaMemcpyAsync(out, o, (size_t)steps * B * H * 2, cudaMemcpyDeviceToHost, c->stream));
        if (stop) CK(cudaMemcpyAsync(stop, sp, (size_t)steps * B * 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaStreamSynchronize(c->stream));
        if ((rc = check_dev_err(c))) return rc;
    }
    return MING_OK;
}

int ming_cuda_cfm_steps(ming_ctx* c, int B, const uint16_t* z, const uint16_t* hist, const uint16_t* y_in,
                        const uint16_t* sde, float cfg, float shift, int step0, int nsteps, uint16_t* y, int kind) {
    if (!c || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    const ming_cfg& f = c->cfg;
    if (f.dit_mode == MING_DIT_NONE) return fail(MING_ERR_INVALID, "no flow head configured");
    if (B < 1 || B > f.dit_max_batch) return fail(MING_ERR_INVALID, "flow batch out of range");
    if (step0 < 0 || nsteps < 1 || step0 + nsteps > 10) return fail(MING_ERR_INVALID, "Euler step range out of [0, 10)");
    const bool ada = f.dit_mode == MING_DIT_ADALN;
    if (!z || !y_in || !y || (!ada && !hist)) return fail(MING_ERR_INVALID, "null argument");
    CK(cudaSetDevice(c->device));
    const int LAT = f.dit_latent, F = f.dit_frames, CD = f.dit_cond_dim;
    int rc;
    // inputs: z rows then zeros (the unconditional half), hist, y, sde
    CK(cudaMemsetAsync(c->f_zc + (size_t)B * CD, 0, (size_t)B * CD * 2, c->stream));
    if ((rc = copy_in(c, c->f_zc, z, (size_t)B * CD * 2, kind))) return rc;
    if (!ada && (rc = copy_in(c, c->f_hist, hist, (size_t)B * LAT * 2, kind))) return rc;
    if ((rc = copy_in(c, c->f_y, y_in, (size_t)B * F * LAT * 2, kind))) return rc;
    if (sde && (rc = copy_in(c, c->f_sde, sde, (size_t)10 * B * F * LAT * 2, kind))) return rc;
    if (cfg != c->cfm_cfg || shift != c->cfm_shift) {  // scalars are baked into the graphs
        for (auto& kv : c->cfm_graphs) cudaGraphExecDestroy(kv.second);
        c->cfm_graphs.clear();
        c->cfm_cfg = cfg;
        c->cfm_shift = shift;
    }
    const int key = ((B * 2 + (sde ? 1 : 0)) * 16 + step0) * 16 + nsteps;
    auto it = c->cfm_graphs.find(key);
    if (it == c->cfm_graphs.end()) {
        cudaGraph_t g;
        CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        if (ada) cfm_ada_enqueue(c, B, sde != nullptr, cfg, shift, step0, nsteps);
        else cfm_token_enqueue(c, B, sde != nullptr, cfg, shift, step0, nsteps);
        cudaError_t ce = cudaStreamEndCapture(c->stream, &g);
        if (ce != cudaSuccess) return fail(MING_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
        cudaGraphExec_t ge;
        ce = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) return fail(MING_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
        it = c->cfm_graphs.emplace(key, ge).first;
    }
    CK(cudaGraphLaunch(it->second, c->stream));
    if ((rc = copy_out(c, y, c->f_y, (size_t)B * F * LAT * 2, kind))) return rc;
    if (kind == MING_PTR_HOST) CK(cudaStreamSynchronize(c->stream));
    return MING_OK;
}

int ming_cuda_cfm_sample(ming_ctx* c, int B, const uint16_t* z, const uint16_t* hist, const uint16_t* noise,
                         const uint16_t* sde, float cfg, float shift, uint16_t* y, int kind) {
    return ming_cuda_cfm_steps(c, B, z, hist, noise, sde, cfg, shift, 0, 10, y, kind);
}

int ming_cuda_aggregate(ming_ctx* c, int B, const uint16_t* latent, uint16_t* out, int kind) {
    if (!c || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    const ming_cfg& f = c->cfg;
    if (!c->agg_proj_on && c->agg.empty()) return fail(MING_ERR_INVALID, "no aggregator configured");
    if (B < 1 || B > f.dit_max_batch || !latent || !out) return fail(MING_ERR_INVALID, "bad argument");
    CK(cudaSetDevice(c->device));
    const int frames = c->agg_proj_on ? f.dit_frames : 1;
    int rc;
    if ((rc = copy_in(c, c->a_lat, latent, (size_t)B * frames * f.dit_latent * 2, kind))) return rc;
    if ((rc = agg_enqueue(c, B, c->a_lat))) return rc;
    CK(cudaGetLastError());
    if ((rc = copy_out(c, out, c->a_out, (size_t)B * f.hidden * 2, kind))) return rc;
    if (kind == MING_PTR_HOST) CK(cudaStreamSynchronize(c->stream));
    return MING_OK;
}

int ming_cuda_get_stream(ming_ctx* c, void** s) {
    if (!c || !s) return fail(MING_ERR_INVALID, "null argument");
    *s = c->stream;
    return MING_OK;
}

int ming_cuda_step_kernels(ming_ctx* c, int B, int* n) {
    if (!c || !n) return fail(MING_ERR_INVALID, "null argument");
    if (!c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    if (B < 1 || B > c->cfg.max_batch) return fail(MING_ERR_INVALID, "batch size out of range");
    // persistent: one launch; per-kernel: step_begin + per layer (4 linears +
    // attention [+ split combine]) + final, mirroring run_linear's dispatch
    if (c->mega_on && B <= MG_MAXB) {
        *n = 1;
        return MING_OK;
    }
    int lin = 2;  // staged: prologue kernel + linear
    if (B <= 64 && c->lin.err && bulk_enabled()) lin = 1;
    else if (B <= 8) lin = 1;
    const int attn = c->nsplit <= 8 ? 1 : 2;
    *n = 1 + (4 * lin + attn) * c->cfg.layers + 1;
    return MING_OK;
}

int ming_cuda_sync(ming_ctx* c) {
    if (!c) return fail(MING_ERR_INVALID, "null context");
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaGetLastError());
    return check_dev_err(c);
}

int ming_cuda_destroy(ming_ctx* c) {
    if (!c) return MING_OK;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->gen_out) cudaFree(c->gen_out);
    if (c->gen_stop) cudaFree(c->gen_stop);
    if (c->err_host) cudaFreeHost(c->err_host);
    delete c;
    return MING_OK;
}

int ming_cuda_kv_read(ming_ctx* c, int s, int layer, int pos0, int n, uint16_t* k, uint16_t* v) {
    if (!c || !c->finalized || !k || !v) return fail(MING_ERR_INVALID, "bad argument");
    int rc = check_seq(c, s);
    if (rc) return rc;
    if (layer < 0 || layer >= c->cfg.layers || pos0 < 0 || n < 0 || pos0 + n > c->seqs[s].len)
        return fail(MING_ERR_INVALID, "range out of bounds");
    CK(cudaStreamSynchronize(c->stream));
    const int KH = c->cfg.kv_heads;
    for (int p = pos0; p < pos0 + n; p++) {
        const int page = c->bt_host[(size_t)s * c->bt_ld + p / PAGE];
        for (int h = 0; h < KH; h++)
            for (int w = 0; w < 2; w++) {
                const size_t off = ((((size_t)page * c->cfg.layers + layer) * 2 + w) * KH + h) * (PAGE * 64) + (p % PAGE) * 64;
                uint16_t* dst = (w == 0 ? k : v) + ((size_t)h * n + (p - pos0)) * 64;
                CK(cudaMemcpy(dst, c->pool + off, 128, cudaMemcpyDeviceToHost));
            }
    }
    return MING_OK;
}

int ming_cuda_kv_write(ming_ctx* c, int s, int layer, int pos0, int n, const uint16_t* k, const uint16_t* v) {
    if (!c || !c->finalized || !k || !v) return fail(MING_ERR_INVALID, "bad argument");
    int rc = check_seq(c, s);
    if (rc) return rc;
    if (layer < 0 || layer >= c->cfg.layers || pos0 < 0 || n < 1 || pos0 > c->seqs[s].len)
        return fail(MING_ERR_INVALID, "range out of bounds");
    CK(cudaSetDevice(c->device));
    if ((rc = ensure_pages(c, s, pos0, pos0 + n))) return rc;
    const int KH = c->cfg.kv_heads;
    const size_t bytes = (size_t)KH * n * HD * 2;
    uint16_t* d = nullptr;
    CK(cudaMalloc(&d, 2 * bytes));
    cudaError_t e = cudaMemcpyAsync(d, k, bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d + bytes / 2, v, bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        kv_write_kernel<<<dim3(n, KH, 2), HD, 0, c->stream>>>(KvDev{c->pool, c->bt, c->bt_ld, c->cfg.layers, KH}, s, layer, pos0,
                                                            n, d, d + bytes / 2);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(d);
    if (e != cudaSuccess) return fail(MING_ERR_CUDA, std::string("kv_write: ") + cudaGetErrorString(e));
    if (pos0 + n > c->seqs[s].len) {
        c->seqs[s].len = pos0 + n;
        CK(cudaMemcpyAsync(c->seq_len + s, &c->seqs[s].len, 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaStreamSynchronize(c->stream));
    }
    return MING_OK;
}

int ming_cuda_unpack_linear(ming_ctx* c, const char* name, float* out) {
    if (!c || !c->finalized || !name || !out) return fail(MING_ERR_INVALID, "bad argument");
    for (PackedLin* pl : c->all_lins) {
        for (size_t si = 0; si < pl->src_names.size(); si++) {
            if (pl->src_names[si] != name) continue;
            const int K = pl->w.K, nrow = pl->w.ntiles * 16;
            float* d = nullptr;
            CK(cudaMalloc(&d, (size_t)nrow * K * 4));
            unpack_tiles_kernel<<<dim3(pl->w.ntiles, K / 64), 32, 0, c->stream>>>(pl->w, d);
            std::vector<float> h((size_t)nrow * K);
            cudaError_t e = cudaMemcpyAsync(h.data(), d, h.size() * 4, cudaMemcpyDeviceToHost, c->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
            cudaFree(d);
            if (e != cudaSuccess) return fail(MING_ERR_CUDA, std::string("unpack: ") + cudaGetErrorString(e));
            for (int i = 0; i < nrow; i++)
                if (pl->rows[i].src == (int)si)
                    std::memcpy(out + (size_t)pl->rows[i].row * K, h.data() + (size_t)i * K, (size_t)K * 4);
            return MING_OK;
        }
    }
    return fail(MING_ERR_INVALID, std::string("no packed linear holds ") + name);
}

// Diagnostics: copies the persistent kernel's phase trace (MING_MEGA_TRACE=1):
// [C][layers][MG_TRACE = 96] clock64 stamps of the last step (slot meanings
// beside MG_TRACE). Returns the CTA
// count in *n. Without it, the per-kernel step's launch trace (MING_KTRACE=1):
// [160 slots][1024 CTAs][8] globaltimer stamps, *n = -(slots used).
extern "C" int ming_cuda_debug_trace(ming_ctx* c, long long* out, int cap, int* n) {
    if (!c || !n) return fail(MING_ERR_INVALID, "null argument");
    *n = 0;
    if (!c->mega_on || !c->mega.trace) {
        // the per-kernel step's launch trace (MING_KTRACE=1): [slot][CTA][8] globaltimer stamps
        if (!c->ktrace) return MING_OK;
        const size_t cnt = (size_t)KT_SLOTS * KT_CTAS * 8;
        if ((size_t)cap < cnt) return fail(MING_ERR_INVALID, "trace buffer too small");
        CK(cudaStreamSynchronize(c->stream));
        CK(cudaMemcpy(out, c->ktrace, cnt * 8, cudaMemcpyDeviceToHost));
        *n = -c->ktrace_used;  // negative: launch-trace slots
        return MING_OK;
    }
    const size_t cnt = (size_t)c->mega.C * c->cfg.layers * MG_TRACE;
    if ((size_t)cap < cnt) return fail(MING_ERR_INVALID, "trace buffer too small");
    CK(cudaStreamSynchronize(c->stream));
    CK(cudaMemcpy(out, c->mega.trace, cnt * 8, cudaMemcpyDeviceToHost));
    *n = c->mega.C;
    return MING_OK;
}

int ming_cuda_flow_temb(ming_ctx* c, uint16_t* te) {
    if (!c || !c->finalized || !te) return fail(MING_ERR_INVALID, "bad argument");
    if (!c->temb) return fail(MING_ERR_INVALID, "no flow head configured");
    CK(cudaMemcpy(te, c->temb, (size_t)10 * c->cfg.dit_hidden * 2, cudaMemcpyDeviceToHost));
    return MING_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------
// Allocation-free decode step
// ---------------------------------------------------------------------
//
// Some callers cannot allocate device memory while they decode: a host
// real-time audio thread must not block in cudaMalloc (which can synchronize
// the whole device), and a process whose device memory is budgeted by another
// runtime gets its cudaMalloc calls refused once the budget is spent. For them
// ming_cuda_lm_decode_noalloc runs one decode step without any device
// allocation: it launches the per-kernel decode sequence directly (no CUDA
// graph is instantiated, which allocates on first use for each batch size)
// and keeps its only scratch, the split-K attention partials, in the
// fixed-size array below instead of a context buffer.

// Most scratch one call may use: the attention partials of B rows,
// B x (max_ctx / 256) splits x heads x 66 f32. 4 MiB covers 32 rows at the
// default 4096 positions (1.9 MB). Every GPU that loads this library holds the
// array until the process exits.
constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)4 << 20;
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {

std::mutex g_noalloc_mu;
constexpr int NOALLOC_MAX_DEVICES = 64;
float* g_noalloc_addr[NOALLOC_MAX_DEVICES] = {};  // device address of the array, per device

// The array's device address on `device` (which must be current). In host
// code `g_noalloc_scratch` names a host-side stand-in, not device memory, so
// the address comes from cudaGetSymbolAddress, once per device.
int noalloc_scratch(int device, float** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (device < 0 || device >= NOALLOC_MAX_DEVICES) return fail(MING_ERR_INVALID, "device index out of range");
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return fail(MING_ERR_CUDA, std::string("scratch address: ") + cudaGetErrorString(e));
        g_noalloc_addr[device] = static_cast<float*>(p);
    }
    *out = g_noalloc_addr[device];
    return MING_OK;
}

}  // namespace

extern "C" int ming_cuda_lm_decode_noalloc(ming_ctx* c, int B, const int* ids, const uint16_t* x, uint16_t* out,
                                           float* stop, int kind) {
    if (!c || !c->finalized) return fail(MING_ERR_INVALID, "context not finalized");
    if (c->cfg.layers < 1) return fail(MING_ERR_INVALID, "no LM configured");
    if (!ids || !x) return fail(MING_ERR_INVALID, "null argument");
    if (B < 1 || B > c->cfg.max_batch) return fail(MING_ERR_INVALID, "batch size out of range");
    const ming_cfg& f = c->cfg;
    // o_proj combines the attention splits in its prologue, which keeps (max,
    // 1/sum) of every (row, head) in the linear kernels' 32-float per-row
    // scratch: 2 x heads must fit in it
    if (2 * f.heads > 32) return fail(MING_ERR_INVALID, "allocation-free decode supports at most 16 query heads");
    const size_t need = (size_t)B * c->nsplit * f.heads * PART_STRIDE * sizeof(float);
    if (need > NOALLOC_SCRATCH_BYTES)
        return fail(MING_ERR_INVALID, "allocation-free decode: " + std::to_string(B) + " rows at max_ctx " +
                                          std::to_string(f.max_ctx) + " need " + std::to_string(need) +
                                          " bytes of attention scratch, more than its fixed " +
                                          std::to_string(NOALLOC_SCRATCH_BYTES) + " bytes");
    CK(cudaSetDevice(c->device));
    float* part = nullptr;
    int rc = noalloc_scratch(c->device, &part);
    if (rc) return rc;
    if ((rc = prepare_rows(c, B, ids, 1))) return rc;
    const int H = f.hidden;
    cudaStream_t s = c->stream;
    uint16_t* null_out = nullptr;
    float* null_stop = nullptr;
    CK(cudaMemcpyAsync(c->out_cell, &null_out, sizeof(void*), cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(c->stop_cell, &null_stop, sizeof(void*), cudaMemcpyHostToDevice, s));
    if ((rc = copy_in(c, c->x, x, (size_t)B * H * 2, kind))) return rc;
    // the per-kernel step (the same launches as the captured decode graph),
    // with the attention partials in the shared scratch array: every split a
    // row reads is written earlier in the same layer, so nothing in it needs
    // clearing between calls
    launch_step_begin(step_dev(c), B, s);
    RowsDev rd{c->row_seq, c->row_pos};
    KvDev kv{c->pool, c->bt, c->bt_ld, f.layers, f.kv_heads};
    for (int l = 0; l < f.layers; l++) {
        auto& L = c->layers[l];
        run_linear(c, L.qkv.w, ProRms{c->x, L.ln1, f.hidden, f.hidden, f.rms_eps, 0, nullptr, L.ln1_unit},
                   EpiQKV{L.qkv.w.bias, c->q, kv, rd, l, f.heads, f.kv_heads, c->log2_theta}, B, s);
        AttnArgs aa{c->q, part, kv, rd, l, f.heads, f.kv_heads, c->nsplit, 1};
        aa.tmap = &c->kv_tmap;
        aa.err = c->dev_err;
        CK(launch_attn(aa, B, s));
        run_linear(c, L.o.w, ProAttn{part, rd, c->nsplit, f.heads, 0, nullptr}, EpiResidual{c->x, c->x1, nullptr, f.hidden}, B,
                   s);
        run_linear(c, L.gu.w, ProRms{c->x1, L.ln2, f.hidden, f.hidden, f.rms_eps, 0, nullptr, L.ln2_unit}, EpiSwiGLU{c->h, f.ff}, B, s);
        run_linear(c, L.down.w, ProPlain{c->h, f.ff, 0}, EpiResidual{c->x1, c->x, nullptr, f.hidden}, B, s);
    }
    launch_final(FinalArgs{c->x, c->norm, c->stop_w, c->stop_b, c->z, c->stop, c->x, step_dev(c), H, 0, 1, f.rms_eps}, B, s);
    CK(cudaGetLastError());
    for (int i = 0; i < B; i++) c->seqs[ids[i]].len += 1;
    if ((rc = copy_out(c, out, c->z, (size_t)B * H * 2, kind))) return rc;
    if ((rc = copy_out(c, stop, c->stop, (size_t)B * 4, kind))) return rc;
    if (kind == MING_PTR_HOST) {
        // The decode-batch linears give up on a weight copy that never lands
        // (a bounded wait) and set the device error flag instead of hanging:
        // read it back with the outputs, as ming_cuda_lm_decode does, so a
        // step that gave up is reported here and not blamed on a later call.
        // With device pointers the flag is read by the next ming_cuda_sync.
        if (c->err_host && c->dev_err) {
            CK(cudaMemcpyAsync(c->err_host, c->dev_err, 4, cudaMemcpyDeviceToHost, s));
            CK(cudaStreamSynchronize(s));
            if (*c->err_host) return check_dev_err(c);
        } else {
            CK(cudaStreamSynchronize(s));
            if ((rc = check_dev_err(c))) return rc;
        }
    }
    return MING_OK;
}
