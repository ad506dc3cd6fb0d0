// mega.cuh — the decode step as one persistent kernel (one CTA per SM).
//
// Why: at batch 1 a 4-bit decode step moves ~205 MB, ~31 us of HBM time at the
// measured 6.5 TB/s, but it is a chain of 24 x 5 dependent GEMV/attention
// phases. Launching each phase as a kernel costs microseconds of launch and
// ramp per phase; here every phase hands off through global memory inside one
// launch, and weight streaming never waits on the chain.
//
// Layout of the work (C = number of CTAs, one per SM):
//   * each GEMV phase's packed tiles (pack.h) are cut into contiguous ranges of
//     64-wide groups, one per CTA (P0 q|k|v, P2 o_proj and P4 down split K;
//     P3 gate|up is cut at whole tiles so a CTA finishes its SwiGLU features
//     itself), so the bytes each CTA streams are balanced;
//   * a producer warp streams the CTA's ranges, layer after layer, with
//     cp.async.bulk into a shared-memory ring guarded by mbarriers, running
//     ahead by the ring's capacity (several layers at 4 bits), together with
//     each layer's norm weights and q|k|v bias;
//   * MG_CWARPS (8) consumer warps run mma.sync on the ring; split-K sums are
//     reduced with red.global.add.u64 on int64 fixed-point accumulators
//     (integer addition is associative: the result is bit-deterministic);
//   * every contribution also adds 2^56, so the top byte of an accumulator
//     counts its contributors: a reader knows a value is complete when that
//     count equals the tile's number of contributing CTAs (static). No writer
//     fence and no completion counter; one thread per CTA first waits for a
//     hint word, then every thread loads its values once and re-polls only
//     the rare incomplete one. SwiGLU outputs are 64-bit words carrying the
//     step's tag beside the bf16 value;
//   * every CTA keeps the residual stream of its rows in shared memory and
//     applies the reference's epilogue math (bias, bf16 rounding, RoPE,
//     residual, SwiGLU) where the values are consumed;
//   * attention is split by (row, query head, 128-position chunk); a chunk's
//     K/V rows are prefetched with cp.async before the CTA waits for q; its
//     (max, sum, P.V) partials carry the step's epoch in each 64-bit word,
//     and the chunk holding the new position combines them with its own and
//     publishes the head's 64 outputs (tagged words) for o_proj.
// Every wait is bounded: on timeout the kernel records an error code, waits
// (bounded) for its own copies in flight and returns.
#pragma once

#include "lm.cuh"

namespace ming {

constexpr int MG_CWARPS = 8;                      // consumer warps
constexpr int MG_THREADS = (MG_CWARPS + 1) * 32;  // + one producer warp
constexpr int MG_CT = MG_CWARPS * 32;             // consumer threads
constexpr int MG_NQ = MG_CT / 64;                 // groups of 64 threads (one per head dim) in the attention combine
static_assert(MG_CT >= 128 && MG_CT % 64 == 0, "consumer threads: whole 64-thread groups, at least one per chunk position");
constexpr int MG_MAXB = 4;                        // rows per step (mma n-tile of 8, half used)
constexpr int MG_ATT_CH = 128;                    // positions per attention item
constexpr int MG_PART = 2 + HD;                   // m, l, acc[64] per attention partial
constexpr int MG_NPH = 4;                         // GEMV phases: P0 qkv, P2 o, P3 gate/up, P4 down
constexpr int MG_FIX = 32;                        // fraction bits of the fixed-point accumulators
constexpr int MG_MAX_STAGE = 32;                  // most 64-groups of activations one CTA stages per phase
// clock64 stamp slots per (CTA, layer) when tracing: 0-9 phase boundaries,
// 10-35 sub-steps of the four GEMV phases, 36-39 attention, 40-55 the end of
// each of the first 8 warps' runs in gate|up and down, 56-63 their first
// gate|up slot in hand, 64-87 the end of their split-K reductions in q|k|v,
// o_proj and down, 88-90 an attention item's q|k|v in hand, pages landed,
// start
constexpr int MG_TRACE = 96;
enum { MG_ACC_QKV = 0, MG_ACC_X1 = 1, MG_ACC_X2 = 2, MG_NACC = 3 };
constexpr int MG_MAX_TILES = 128;                 // most tiles of a split-K phase (q|k|v, o_proj, down)

struct MegaPhase {
    const int* cta_g0;  // [C + 1]: CTA c owns flattened groups [cta_g0[c], cta_g0[c+1])
    const int* tcount;  // [tiles]: CTAs contributing to each tile (split-K phases), or null
    int tiles, gpt;
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
    unsigned long long* acc;   // [2 parity][layers][MG_NACC][MG_MAXB][acc_w] int64 fixed point
    int acc_w;
    uint64_t* hbuf;            // [layers][MG_MAXB][FF] SwiGLU outputs: step tag << 32 | bf16
    uint64_t* attn;            // [B][heads][max_splits][MG_PART] tagged attention partials
    uint64_t* comb;            // [MG_MAXB][heads][64] tagged combined attention outputs (the o_proj input)
    const uint16_t* x_in;      // [B][H] step input
    uint16_t* z;               // [B][H] post-norm hidden
    uint16_t* feed;            // [B][H] copy of z (next step's input)
    float* stop;               // [B]
    uint16_t* const* out_cell; // per-step output slots (generate) or null
    float* const* stop_cell;
    int* counter;              // [2]: epoch, generate step index
    int* err;                  // error code (0 = ok)
    long long* trace;          // optional [C][layers][MG_TRACE] clock64 stamps (null = off)
    int layers, H, FF, heads, kvh, fmt, C, B, max_splits, gps, cb, nslots, slot_bytes;
    float log2_theta, eps;
};

// Host side (mega.cu)
int mega_smem_bytes(int nslots, int slot_bytes, int H, int lp_bytes);
cudaError_t launch_mega(const MegaDev& a, int smem, cudaStream_t s);

}  // namespace ming
