// pack.h — host-side repacking of linear weights into the tile layout the
// kernels stream.
//
// A packed linear is a sequence of 16-row tiles; tile row r holds some source
// row (feature) chosen by the caller, so an epilogue finds the pairs it needs
// (RoPE halves, rotary neighbours, gate/up) in one thread. Each tile is K/64
// chunks, one per 64-wide group of the reduction dimension:
//
//   fmt 4 : 512 B codes  [lane 0..31][4 words]   + 64 B scales  = 576 B
//   fmt 8 : 1024 B codes [2][lane][4 words]       + 64 B scales  = 1088 B
//   fmt 16: 2048 B       [kstep 0..3][lane][4 words]             = 2048 B
//
// The word a lane holds for one 16-wide k-step carries exactly its mma.sync
// A-fragment (rows g, g+8; k = 2t, 2t+1, 2t+8, 2t+9 with g = lane/4,
// t = lane%4), in the order common.cuh's dq4/dq8 unpack. Scales: 8 entries of
// (scale[g], bias[g], scale[g+8], bias[g+8]) bf16 — the MLX affine group
// parameters of the tile's rows for that group.
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

namespace ming {

// One source weight matrix in the reference's layout (host memory).
struct LinearSrc {
    int fmt = 16;  // 16 (bf16), 8 or 4 (MLX affine)
    int out = 0, in = 0, group = 64;
    const uint16_t* w = nullptr;       // bf16 [out][in]
    const uint32_t* q = nullptr;       // uint32 [out][in*fmt/32]
    const uint16_t* scales = nullptr;  // bf16 [out][in/group]
    const uint16_t* biases = nullptr;  // bf16 [out][in/group]
    const uint16_t* bias = nullptr;    // bf16 [out] linear bias, optional
};

struct RowRef {
    int src = -1;  // index into the source list; -1 = zero padding row
    int row = 0;
};

inline int chunk_bytes(int fmt) { return fmt == 4 ? 576 : (fmt == 8 ? 1088 : 2048); }

// Packs rows (size 16 * ntiles) into tiles. Returns "" or an error message.
std::string pack_tiles(const std::vector<LinearSrc>& srcs, const std::vector<RowRef>& rows, int fmt, int K,
                       std::vector<uint8_t>& out, std::vector<float>& bias_out);

}  // namespace ming
