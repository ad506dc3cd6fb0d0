// mega.cuh — the decode step as one persistent kernel (one CTA per SM).
//
// Why: at batch 1 a 4-bit decode step moves ~205 MB, ~31 us of HBM time at the
// measured 6.5 TB/s, but it is a chain of 24 x 5 dependent GEMV/attention
// phases. Launching each phase as a kernel costs microseconds of launch and
// ramp per phase; here every phase hands off through global memory inside one
// launch, and weight streaming never waits on the chain.
//
// Layout of the work (C = number of CTAs, one per SM):
//   * every GEMV phase (P0 q|k|v, P2 o_proj, P3 gate|up, P4 down) is split by
//     64-wide groups of its reduction dimension: CTA c owns the contiguous
//     range [c*G/C, (c+1)*G/C) of the phase's G = tiles x groups-per-tile
//     chunks, i.e. a contiguous byte range of the packed tile buffer
//     (pack.h), so bytes per CTA are balanced to one group;
//   * a producer warp streams the CTA's ranges, layer after layer, with
//     cp.async.bulk into a shared-memory ring guarded by mbarriers; it runs
//     ahead by the ring's capacity (several layers at 4 bits);
//   * 8 consumer warps run the mma.sync tiles on the ring and write one f32
//     partial per (tile, CTA) — the split-K partial sums;
//   * the consumers of a phase reduce the partials of the tiles they need in a
//     fixed order (deterministic) and apply the epilogue math of the reference
//     (bias, bf16 rounding, RoPE, residual, SwiGLU) in their prologue; every
//     CTA keeps the whole residual stream of its rows in shared memory and
//     updates it from the o_proj / down partials, so no residual is published;
//   * attention (P1) is split by (row, kv head, 128-position chunk); the chunk's
//     K/V pages are prefetched with cp.async before the CTA waits for q.
// Hand-offs: every published value carries the step's epoch tag in the same
// 64-bit word (single-copy atomic), so a consumer polls the data itself — no
// flag, no fence. A consumer issues all loads of a batch before checking any
// tag (one L2 round trip per batch, not per word). Every wait is bounded; on
// timeout the kernel records an error code and returns.
#pragma once

#include "lm.cuh"

namespace ming {

constexpr int MG_CWARPS = 8;                      // consumer warps
constexpr int MG_THREADS = (MG_CWARPS + 1) * 32;  // + one producer warp
constexpr int MG_MAXB = 4;                        // rows per step (mma n-tile of 8, half used)
constexpr int MG_ATT_CH = 128;                    // positions per attention item
constexpr int MG_PART = 2 + HD;                   // m, l, acc[64] per attention partial
constexpr int MG_NPH = 4;                         // GEMV phases: P0 qkv, P2 o, P3 gate/up, P4 down

struct MegaPhase {
    const int* cta_g0;   // [C + 1]: CTA c owns flattened groups [cta_g0[c], cta_g0[c+1])
    const int* tile_c0;  // [tiles]: first CTA covering the tile (partial slot = c - tile_c0[t])
    uint64_t* part;      // [layers][tiles][slots][16][B] tagged f32 partials
    int tiles, gpt, slots;
};

struct MegaDev {
    const uint8_t* const* wbase;  // [layers * 4] packed tile buffers (P0, P2, P3, P4)
    MegaPhase ph[MG_NPH];
    // per-layer parameters, one contiguous block per layer streamed to shared
    // memory with the weights: ln1 [H] bf16 | ln2 [H] bf16 | q|k|v bias
    // [(heads + 2 kvh) * 64] f32 in packed row order
    const uint8_t* lparams;
    int lp_bytes;
    const uint16_t* norm;      // final norm [H]
    const uint16_t* stop_w;    // [2][H]
    const uint16_t* stop_b;    // [2]
    KvDev kv;
    int* seq_len;              // [max_seqs]
    const int* row_seq;        // [B]
    uint64_t* attn;            // [B][heads][max_splits][MG_PART] tagged attention partials
    const uint16_t* x_in;      // [B][H] step input
    uint16_t* z;               // [B][H] post-norm hidden
    uint16_t* feed;            // [B][H] copy of z (next step's input)
    float* stop;               // [B]
    uint16_t* const* out_cell; // per-step output slots (generate) or null
    float* const* stop_cell;
    int* counter;              // [2]: epoch, generate step index
    int* err;                  // error code (0 = ok)
    long long* trace;          // optional [C][layers][32] clock64 stamps at phase ends (null = off)
    int layers, H, FF, heads, kvh, fmt, C, B, max_splits, gps, cb, nslots, slot_bytes;
    float log2_theta, eps;
};

// Host side (mega.cu)
// Shared memory the kernel needs (bytes) for a ring of nslots x slot_bytes.
int mega_smem_bytes(int nslots, int slot_bytes, int H, int lp_bytes);
constexpr int MG_MAX_STAGE = 32;  // most 64-groups of activations one CTA stages per phase
cudaError_t launch_mega(const MegaDev& a, int smem, cudaStream_t s);

}  // namespace ming
