// runtime.h — internal to the library: the context behind include/ming_cuda.h
// and the host helpers its translation units share (runtime.cu: weights, KV
// pages, decode graphs, flow head; loop.cu: the sampling loop and its request
// scheduler).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <map>
#include <string>
#include <vector>

#include "../../include/ming_cuda.h"
#include "mega.cuh"
#include "pack.h"

namespace ming {
namespace rt {

// Records m as the calling thread's last error (ming_cuda_last_error) and
// returns code.
int fail(int code, const std::string& m);

// Returns MING_ERR_CUDA with the failing call's text when a CUDA call fails.
#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            return ::ming::rt::fail(MING_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

struct HostTensor {
    int dtype = 0;
    std::vector<int64_t> shape;
    std::vector<uint8_t> data;
    int64_t dim(int i) const { return i < (int)shape.size() ? shape[i] : 1; }
};

// A device allocation freed with the context.
struct DevMem {
    std::vector<void*> ptrs;
    ~DevMem() {
        for (void* p : ptrs) cudaFree(p);
    }
    template <class T>
    T* alloc(size_t count, int* rc) {
        void* p = nullptr;
        if (count == 0) count = 1;
        cudaError_t e = cudaMalloc(&p, count * sizeof(T));
        if (e != cudaSuccess) {
            *rc = fail(MING_ERR_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
            return nullptr;
        }
        cudaMemset(p, 0, count * sizeof(T));
        ptrs.push_back(p);
        return static_cast<T*>(p);
    }
};

struct PackedLin {
    PackedW w;
    std::vector<std::string> src_names;  // weight names of the sources
    std::vector<RowRef> rows;
    std::vector<int> src_out, src_in;
};

struct DitBlockW {
    PackedLin ada, qkv, o, ff1, ff2;
    uint16_t* norm1 = nullptr;
    uint16_t* norm2 = nullptr;
};

struct SeqInfo {
    bool live = false;
    int len = 0;
};

}  // namespace rt
}  // namespace ming

struct ming_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    ming_cfg cfg{};
    bool finalized = false;
    std::map<std::string, ming::rt::HostTensor> staged;
    ming::rt::DevMem mem;
    std::vector<ming::rt::PackedLin*> all_lins;

    // LM
    struct Layer {
        ming::rt::PackedLin qkv, o, gu, down;
        uint16_t* ln1 = nullptr;
        uint16_t* ln2 = nullptr;
        bool ln1_unit = false, ln2_unit = false;  // every gain is exactly 1
    };
    std::vector<Layer> layers;
    uint16_t* norm = nullptr;
    uint16_t* stop_w = nullptr;
    uint16_t* stop_b = nullptr;
    float log2_theta = 0;

    // KV
    uint16_t* pool = nullptr;
    int* bt = nullptr;
    int bt_ld = 0;
    std::vector<int> bt_host;
    std::vector<int> free_pages;
    std::vector<ming::rt::SeqInfo> seqs;

    // activations / step state
    int maxr = 0, nsplit = 0;
    uint16_t *x = nullptr, *x1 = nullptr, *q = nullptr, *h = nullptr, *z = nullptr;
    uint16_t* att = nullptr;  // [maxr][heads * 64] combined attention output (o_proj input)
    ming::LinScratch lin;     // staged activations of linears over more than 8 rows
    float* stop = nullptr;
    float* part = nullptr;
    int *seq_len = nullptr, *row_seq = nullptr, *row_pos = nullptr, *step_counter = nullptr;
    uint16_t** out_cell = nullptr;
    float** stop_cell = nullptr;
    std::vector<int> row_seq_host;
    std::map<int, cudaGraphExec_t> decode_graphs;
    // persistent decode kernel (batches of up to MG_MAXB rows)
    bool mega_on = false;
    ming::MegaDev mega{};
    int mega_smem = 0;
    CUtensorMap kv_tmap;  // the page pool as attn_partial_kernel's TMA source (lm.cuh)
    int* dev_err = nullptr;
    int* err_host = nullptr;  // pinned: the device error flag read back with a call's outputs
    bool cells_null = false;  // out_cell / stop_cell known to hold null (decode); generate sets them
    // launch trace of the per-kernel step (MING_KTRACE=1): KT_SLOTS launches x
    // KT_CTAS CTAs x 8 globaltimer stamps, slot = launch order in the step
    long long* ktrace = nullptr;
    int ktrace_used = 0;
    int* mega_counter = nullptr;  // [2]: epoch (monotonic), generate step index
    std::function<cudaError_t()> mega_reset;  // clean persistent-kernel state after a device error
    uint16_t* gen_out = nullptr;
    size_t gen_out_elems = 0;
    float* gen_stop = nullptr;
    size_t gen_stop_elems = 0;

    // flow head
    std::vector<ming::rt::DitBlockW> dit;
    ming::rt::PackedLin t_mlp0, t_mlp2, x_emb, c_emb, final_ada, final_lin;
    uint16_t* final_norm = nullptr;
    uint16_t* final_w = nullptr;  // token final linear, raw bf16 [latent][H]
    uint16_t* final_b = nullptr;
    float* inv_freq = nullptr;
    uint16_t* temb = nullptr;  // [10][H]
    float flow_dt[10] = {0}, flow_sq[10] = {0};
    uint16_t *f_z = nullptr, *f_zc = nullptr, *f_hist = nullptr, *f_y = nullptr, *f_sde = nullptr;
    uint16_t *f_ce = nullptr, *f_xh = nullptr, *f_xy = nullptr, *f_rows = nullptr, *f_x1 = nullptr, *f_qkv = nullptr;
    uint16_t *f_att = nullptr, *f_hh = nullptr, *f_sc = nullptr, *f_mod = nullptr;
    float* f_vel = nullptr;
    std::map<int, cudaGraphExec_t> cfm_graphs;  // (B, sde?, step0, nsteps) -> graph
    float cfm_cfg = NAN, cfm_shift = NAN;

    // aggregator
    std::vector<ming::rt::DitBlockW> agg;
    ming::rt::PackedLin agg_x_emb, agg_final;
    // adaLN head: latent -> next LM input (mean over frames, then aggregator.proj)
    ming::rt::PackedLin agg_proj;
    bool agg_proj_on = false;
    uint16_t* a_mean = nullptr;
    uint16_t* agg_cls = nullptr;
    uint16_t* agg_norm = nullptr;
    float* agg_inv_freq = nullptr;
    uint16_t *a_lat = nullptr, *a_rows = nullptr, *a_x1 = nullptr, *a_qkv = nullptr, *a_att = nullptr, *a_hh = nullptr,
             *a_xe = nullptr, *a_out = nullptr;

    // VAE decoder (vae.cu): linears packed with their K doubled ([W | W]) so
    // f32 activations enter as bf16 hi / lo halves; the ISTFT's irfft as a
    // linear with the DFT basis (K tripled: hi, lo and hi parts)
    struct VaeLayer {
        ming::rt::PackedLin qkv, o, gu, down;
        uint16_t* ln1 = nullptr;
        uint16_t* ln2 = nullptr;
    };
    std::vector<VaeLayer> vae;
    ming::rt::PackedLin vae_fc1, vae_head, vae_dft;
    uint16_t* vae_norm = nullptr;
    float* vae_win = nullptr;
    uint16_t *v_lat = nullptr, *v_fc1 = nullptr;
    float *v_x = nullptr, *v_q = nullptr, *v_k = nullptr, *v_v = nullptr, *v_att = nullptr, *v_h = nullptr;
    float *v_head = nullptr, *v_spec = nullptr, *v_frames = nullptr, *v_wave = nullptr;

    ~ming_ctx() {
        for (auto& kv : decode_graphs) cudaGraphExecDestroy(kv.second);
        for (auto& kv : cfm_graphs) cudaGraphExecDestroy(kv.second);
        if (stream) cudaStreamDestroy(stream);
    }
};


namespace ming {
namespace rt {

// Shared host helpers (runtime.cu). All work goes on the context's stream.
// The next launch-trace slot of a step (MING_KTRACE=1) or null.
long long* ktrace_slot(ming_ctx* c);
// A weight from the staged tensors: "<prefix>.weight" bf16, or U32 + .scales
// + .biases; its bias when want_bias.
int lin_src(ming_ctx* c, const std::string& prefix, LinearSrc& s, bool want_bias);
// Packs sources into the kernels' tiles (rows in the given order) on the device.
int upload_packed(ming_ctx* c, const std::vector<LinearSrc>& srcs, const std::vector<std::string>& names,
                  const std::vector<RowRef>& rows, PackedLin& pl);
// A staged tensor copied to the device as is (checked dtype and element count).
int upload_raw(ming_ctx* c, const std::string& name, int dtype, int64_t count, void** out);
const HostTensor* find_staged(ming_ctx* c, const std::string& name);
// A linear in plain row order (tile row r = output 16 t + r), its out dim in *out_dim.
int pack_plain(ming_ctx* c, const std::string& prefix, bool bias, PackedLin& pl, int* out_dim = nullptr);
int check_seq(ming_ctx* c, int s);
// Gives positions [from, to) of sequence s pages; uploads new block-table entries.
int ensure_pages(ming_ctx* c, int s, int from, int to);
// Validates a batch of sequences for `steps` decode steps and uploads row_seq.
int prepare_rows(ming_ctx* c, int B, const int* seq_ids, int steps);
// Reads (and clears) the device error flag; MING_ERR_CUDA if a bounded wait gave up.
int check_dev_err(ming_ctx* c);
// The body of one decode step of B rows (the persistent kernel, or the
// per-kernel layers and final norm): input c->x, outputs c->z, c->stop.
cudaError_t decode_enqueue(ming_ctx* c, int B);
// The flow head's Euler steps [step0, step0 + nsteps) over B conditions, on
// the context's flow buffers (f_zc, f_hist, f_y, f_sde); result in f_y.
int cfm_enqueue(ming_ctx* c, int B, bool with_sde, float cfg, float shift, int step0, int nsteps);
// Model.aggregate of B latents on the device (token mode: the aggregator's
// blocks; adaLN mode: frame mean + aggregator.proj) into c->a_out.
int agg_enqueue(ming_ctx* c, int B, const uint16_t* latent);
// The VAE decoder's weights and buffers (vae.cu), when cfg.vae_layers > 0.
int vae_finalize(ming_ctx* c);
// Returns a sequence's pages to the pool without synchronising: the block
// table reset is queued on the stream, behind every kernel that reads it.
int seq_release(ming_ctx* c, int s);

}  // namespace rt
}  // namespace ming
