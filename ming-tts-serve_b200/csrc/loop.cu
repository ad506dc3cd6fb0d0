// loop.cu — the autoregressive sampling loop on the device, and a request
// scheduler that keeps its rows full (continuous batching).
//
// The reference runs one sequence at a time (sampleLatents,
// src/ming_model.zig:1388-1480; one engine thread and a FIFO of requests,
// src/ming_service.zig:175-206,277-287). Per step it samples the flow head on
// the last hidden state, aggregates the latent into the next LM input, runs
// one LM step and reads the previous hidden state's stop probability back; it
// stops on p > 0.5 after step 3, within min(max_steps, 512 - prompt length)
// steps.
//
// Here up to R sequences share each step. One CUDA graph per row count runs
// the whole step: a prep kernel (each row's condition, history and noise into
// the flow head's buffers), the flow head's 10 Euler steps, the aggregator,
// one LM decode step, and an update kernel that records each row's latent,
// applies the stop rule on the device and advances the row. The host reads
// the rows' stop flags one step behind (the step after is already queued, as
// the reference pipelines), retires finished rows by moving the last active
// row into their place, and admits queued requests into the freed rows
// (their prompt prefills between two steps).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "runtime.h"

using namespace ming;
using namespace ming::rt;

namespace {

constexpr int LOOP_STEPS = 10;  // Euler steps per flow-head sample (FLOW_STEPS)

// Per-row state of the loop on the device (rows 0..B-1 are active).
struct LoopRows {
    uint16_t* z;         // [R][H] LM hidden state that conditions this step's sample
    float* stop;         // [R] its stop probability
    uint16_t* hist;      // [R][LAT] the previous latent (token mode's history)
    int* step;           // [R] step index of the row's request
    int* budget;         // [R] steps the request may take
    int* done;           // [R] 1 once the stop rule or the budget ended it
    int* n_out;          // [R] latents emitted
    unsigned long long* seed;  // [R] noise stream of the request
    const uint16_t** bank;     // [R] replay bank [steps][11][FL] or null (seeded noise)
    uint16_t** out_lat;        // [R] -> [budget][FL]
    uint16_t** out_z;          // [R] -> [budget][H] or null
    float** out_stop;          // [R] -> [budget]
};

// ---- seeded noise: the same SplitMix64 / Box-Muller streams as the test
// harness's generator (one stream per (seed, "loop.noise.<step>"), 11 rows of
// FL values: the start noise, then the 10 SDE draws) ----
constexpr unsigned long long GOLDEN = 0x9E3779B97F4A7C15ull;
__device__ __forceinline__ unsigned long long splitmix(unsigned long long z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// FNV-1a-64 of "loop.noise." followed by the decimal digits of step
__device__ unsigned long long noise_stream(unsigned long long seed, int step) {
    const char pre[] = "loop.noise.";
    unsigned long long h = 0xCBF29CE484222325ull;
    for (int i = 0; pre[i]; i++) h = (h ^ (unsigned char)pre[i]) * 0x100000001B3ull;
    char dig[12];
    int n = 0;
    unsigned v = (unsigned)step;
    do {
        dig[n++] = (char)('0' + v % 10);
        v /= 10;
    } while (v);
    while (n) h = (h ^ (unsigned char)dig[--n]) * 0x100000001B3ull;
    return seed * GOLDEN ^ h;
}
// element e of the stream: Box-Muller pair e / 2 from outputs 2m+1, 2m+2
__device__ uint16_t noise_value(unsigned long long s0, int e) {
    const int m = e >> 1;
    const unsigned long long x1 = splitmix(s0 + (unsigned long long)(2 * m + 1) * GOLDEN);
    const unsigned long long x2 = splitmix(s0 + (unsigned long long)(2 * m + 2) * GOLDEN);
    const double u1 = ((double)(x1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = ((double)(x2 >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double r = sqrt(-2.0 * log(u1)), t = (2.0 * 3.141592653589793) * u2;
    const double v = (e & 1) ? r * sin(t) : r * cos(t);
    return f2bf((float)v);
}

// Each row's condition (z, then a zero row for the unconditional half),
// history and noise into the flow head's input buffers. Grid (B, 12): y = 0
// z and history, y = 1 + j noise row j (0 start noise, 1..10 SDE draws).
__global__ void loop_prep_kernel(LoopRows r, int B, int H, int LAT, int FL, bool token, bool sde, uint16_t* f_zc,
                                 uint16_t* f_hist, uint16_t* f_y, uint16_t* f_sde) {
    const int b = blockIdx.x, j = blockIdx.y - 1, tid = threadIdx.x;
    if (j < 0) {
        for (int i = tid; i < H; i += blockDim.x) {
            f_zc[(size_t)b * H + i] = r.z[(size_t)b * H + i];
            f_zc[(size_t)(B + b) * H + i] = 0;
        }
        if (token)
            for (int i = tid; i < LAT; i += blockDim.x) f_hist[(size_t)b * LAT + i] = r.hist[(size_t)b * LAT + i];
        return;
    }
    if (j > 0 && !sde) return;
    uint16_t* dst = j == 0 ? f_y + (size_t)b * FL : f_sde + ((size_t)(j - 1) * B + b) * FL;
    const int st = r.step[b];
    const uint16_t* bank = r.bank[b];
    if (bank) {
        const uint16_t* src = bank + ((size_t)st * (LOOP_STEPS + 1) + j) * FL;
        for (int i = tid; i < FL; i += blockDim.x) dst[i] = src[i];
    } else {
        const unsigned long long s0 = noise_stream(r.seed[b], st);
        for (int i = tid; i < FL; i += blockDim.x) dst[i] = noise_value(s0, j * FL + i);
    }
}

// After the step: record each live row's latent (and the z / stop that
// produced it), apply the stop rule of sampleLatents (p > 0.5 and step > 3,
// src/ming_model.zig:1467) and the budget, and advance the row: history =
// latent, z = the LM's new hidden state, stop = its probability.
__global__ void loop_update_kernel(LoopRows r, int H, int LAT, int FL, bool token, const uint16_t* f_y, const uint16_t* z_new,
                                   const float* stop_new) {
    const int b = blockIdx.x, tid = threadIdx.x;
    if (r.done[b]) return;  // block-uniform
    const int k = r.step[b];
    const float sp = r.stop[b];
    const uint16_t* lat = f_y + (size_t)b * FL;
    uint16_t* ol = r.out_lat[b] + (size_t)k * FL;
    for (int i = tid; i < FL; i += blockDim.x) ol[i] = lat[i];
    if (r.out_z[b]) {
        uint16_t* oz = r.out_z[b] + (size_t)k * H;
        for (int i = tid; i < H; i += blockDim.x) oz[i] = r.z[(size_t)b * H + i];
    }
    const bool stop = (sp > 0.5f && k > 3) || k + 1 >= r.budget[b];
    __syncthreads();  // every read of this row's z above precedes its update below
    if (tid == 0) {
        r.out_stop[b][k] = sp;
        r.n_out[b] = k + 1;
        if (stop) r.done[b] = 1;
        else {
            r.step[b] = k + 1;
            r.stop[b] = stop_new[b];
        }
    }
    if (stop) return;
    for (int i = tid; i < H; i += blockDim.x) r.z[(size_t)b * H + i] = z_new[(size_t)b * H + i];
    if (token)  // history patch of one frame: the latent just emitted
        for (int i = tid; i < LAT; i += blockDim.x) r.hist[(size_t)b * LAT + i] = lat[FL - LAT + i];
}

// Moves row state src -> dst for each (dst, src) pair, in order (compaction
// after retirements: dst a retired row, src the last live one). One thread
// handles the same elements of every pair, so a row an earlier pair filled
// may be a later pair's source.
__global__ void loop_move_kernel(LoopRows r, const int* pairs, int n, int H, int LAT) {
    for (int p = 0; p < n; p++) {
        const int d = pairs[2 * p], s = pairs[2 * p + 1];
        for (int i = threadIdx.x; i < H; i += blockDim.x) r.z[(size_t)d * H + i] = r.z[(size_t)s * H + i];
        for (int i = threadIdx.x; i < LAT; i += blockDim.x) r.hist[(size_t)d * LAT + i] = r.hist[(size_t)s * LAT + i];
        if (threadIdx.x == 0) {
            r.stop[d] = r.stop[s];
            r.step[d] = r.step[s];
            r.budget[d] = r.budget[s];
            r.done[d] = r.done[s];
            r.n_out[d] = r.n_out[s];
            r.seed[d] = r.seed[s];
            r.bank[d] = r.bank[s];
            r.out_lat[d] = r.out_lat[s];
            r.out_z[d] = r.out_z[s];
            r.out_stop[d] = r.out_stop[s];
        }
    }
}

enum { REQ_QUEUED = 0, REQ_ACTIVE = 1, REQ_DONE = 2 };

struct Request {
    int state = REQ_QUEUED;
    int seq = -1, L = 0, budget = 0, n_out = 0;
    std::vector<uint16_t> embeds;    // until admitted
    std::vector<uint16_t> hist0;     // [LAT] history seed (zeros without a prompt latent)
    std::vector<uint16_t> bank;      // replay bank until admitted (empty: seeded)
    unsigned long long seed = 0;
    bool trace = false;
    uint16_t *d_lat = nullptr, *d_z = nullptr, *d_bank = nullptr;
    float* d_stop = nullptr;
    std::string error;
    void free_device() {
        cudaFree(d_lat);
        cudaFree(d_z);
        cudaFree(d_bank);
        cudaFree(d_stop);
        d_lat = d_z = d_bank = nullptr;
        d_stop = nullptr;
    }
};

}  // namespace

struct ming_loop {
    ming_ctx* c = nullptr;
    int R = 0, H = 0, LAT = 0, FL = 0, cap = 0;
    bool token = true, sde = false;
    ming_sample_params p{};
    float shift = 0.f;
    LoopRows d{};
    int* d_pairs = nullptr;        // [2R] compaction pairs
    void* d_block = nullptr;       // one allocation holding every per-row array
    int* h_flags = nullptr;        // pinned [2][2R]: done, n_out of every row after a step
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool pending[2] = {false, false};
    std::vector<int> rows_at[2];   // row -> request id when that step was queued
    long long nstep = 0;
    std::vector<int> rows;         // row -> request id (active rows, compact)
    std::map<int, Request> reqs;
    std::deque<int> queue;
    int next_id = 0;
    std::map<int, cudaGraphExec_t> graphs;  // row count -> the step's graph
    ~ming_loop() {
        for (auto& g : graphs) cudaGraphExecDestroy(g.second);
        for (auto& q : reqs) q.second.free_device();
        for (cudaEvent_t e : ev)
            if (e) cudaEventDestroy(e);
        if (h_flags) cudaFreeHost(h_flags);
        cudaFree(d_block);
    }
};

namespace {

// The step's work for B rows on the context's stream (captured once per B).
int loop_enqueue(ming_loop* lp, int B) {
    ming_ctx* c = lp->c;
    const ming_cfg& f = c->cfg;
    cudaStream_t s = c->stream;
    loop_prep_kernel<<<dim3(B, LOOP_STEPS + 2), 128, 0, s>>>(lp->d, B, lp->H, lp->LAT, lp->FL, lp->token, lp->sde, c->f_zc,
                                                            c->f_hist, c->f_y, c->f_sde);
    int rc = cfm_enqueue(c, B, lp->sde, lp->p.cfg, lp->shift, 0, LOOP_STEPS);
    if (rc) return rc;
    if ((rc = agg_enqueue(c, B, c->f_y))) return rc;
    CK(cudaMemcpyAsync(c->x, c->a_out, (size_t)B * f.hidden * 2, cudaMemcpyDeviceToDevice, s));
    CK(decode_enqueue(c, B));
    loop_update_kernel<<<B, 128, 0, s>>>(lp->d, lp->H, lp->LAT, lp->FL, lp->token, c->f_y, c->z, c->stop);
    return MING_OK;
}

int loop_graph(ming_loop* lp, int B, cudaGraphExec_t* out) {
    auto it = lp->graphs.find(B);
    if (it != lp->graphs.end()) {
        *out = it->second;
        return MING_OK;
    }
    ming_ctx* c = lp->c;
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = loop_enqueue(lp, B);
    const cudaError_t le = cudaGetLastError();
    const cudaError_t ce = cudaStreamEndCapture(c->stream, &g);
    if (rc || le != cudaSuccess || ce != cudaSuccess) {
        if (ce == cudaSuccess) cudaGraphDestroy(g);
        if (rc) return rc;
        return fail(MING_ERR_CUDA, std::string("loop step capture: ") + cudaGetErrorString(le != cudaSuccess ? le : ce));
    }
    cudaGraphExec_t ge;
    const cudaError_t ie = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) return fail(MING_ERR_CUDA, std::string("loop graph instantiate: ") + cudaGetErrorString(ie));
    lp->graphs[B] = ge;
    *out = ge;
    return MING_OK;
}

// Prefills a queued request into row `row` (queued on the stream: the prompt
// runs between two steps) and seeds the row's state.
int admit(ming_loop* lp, int id, int row) {
    ming_ctx* c = lp->c;
    Request& q = lp->reqs[id];
    const int H = lp->H, L = q.L;
    int rc = ming_cuda_seq_alloc(c, &q.seq);
    if (rc) return rc;
    // every position the request can reach: prompt, budget, and the one step
    // a finished row may still run before the host retires it
    if ((rc = ensure_pages(c, q.seq, 0, L + q.budget + 1))) {
        seq_release(c, q.seq);
        q.seq = -1;
        return rc;
    }
    // the prompt's temporaries are stream-ordered: freed behind the prefill
    // that reads them, without waiting for the step in flight
    uint16_t* d_emb = nullptr;
    uint16_t* d_out = nullptr;
    float* d_pst = nullptr;
    CK(cudaMallocAsync(&d_emb, (size_t)L * H * 2, c->stream));
    CK(cudaMallocAsync(&d_out, (size_t)L * H * 2, c->stream));
    CK(cudaMallocAsync(&d_pst, (size_t)L * 4, c->stream));
    CK(cudaMalloc(&q.d_lat, (size_t)q.budget * lp->FL * 2));
    CK(cudaMalloc(&q.d_stop, (size_t)q.budget * 4));
    if (q.trace) CK(cudaMalloc(&q.d_z, (size_t)q.budget * H * 2));
    if (!q.bank.empty()) {
        CK(cudaMalloc(&q.d_bank, q.bank.size() * 2));
        CK(cudaMemcpyAsync(q.d_bank, q.bank.data(), q.bank.size() * 2, cudaMemcpyHostToDevice, c->stream));
    }
    CK(cudaMemcpyAsync(d_emb, q.embeds.data(), (size_t)L * H * 2, cudaMemcpyHostToDevice, c->stream));
    rc = ming_cuda_lm_prefill(c, q.seq, d_emb, L, d_out, d_pst, MING_PTR_DEVICE);
    if (!rc) {
        // the row's state: z = last prompt hidden state, its stop probability,
        // the history seed, step 0 (pointer-sized fields through one staging copy)
        const LoopRows& r = lp->d;
        CK(cudaMemcpyAsync(r.z + (size_t)row * H, d_out + (size_t)(L - 1) * H, (size_t)H * 2, cudaMemcpyDeviceToDevice,
                           c->stream));
        CK(cudaMemcpyAsync(r.stop + row, d_pst + L - 1, 4, cudaMemcpyDeviceToDevice, c->stream));
        CK(cudaMemcpyAsync(r.hist + (size_t)row * lp->LAT, q.hist0.data(), (size_t)lp->LAT * 2, cudaMemcpyHostToDevice,
                           c->stream));
        const int zero = 0;
        CK(cudaMemcpyAsync(r.step + row, &zero, 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(r.done + row, &zero, 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(r.n_out + row, &zero, 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(r.budget + row, &q.budget, 4, cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(r.seed + row, &q.seed, 8, cudaMemcpyHostToDevice, c->stream));
        const void* ptrs[4] = {q.d_bank, q.d_lat, q.d_z, q.d_stop};
        CK(cudaMemcpyAsync(r.bank + row, &ptrs[0], sizeof(void*), cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(r.out_lat + row, &ptrs[1], sizeof(void*), cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(r.out_z + row, &ptrs[2], sizeof(void*), cudaMemcpyHostToDevice, c->stream));
        CK(cudaMemcpyAsync(r.out_stop + row, &ptrs[3], sizeof(void*), cudaMemcpyHostToDevice, c->stream));
        // the host-side sources above are pageable: each copy is staged before
        // the call returns, so the locals may go out of scope
    }
    cudaFreeAsync(d_emb, c->stream);
    cudaFreeAsync(d_out, c->stream);
    cudaFreeAsync(d_pst, c->stream);
    if (rc) {
        q.free_device();
        seq_release(c, q.seq);
        q.seq = -1;
        return rc;
    }
    q.embeds.clear();
    q.embeds.shrink_to_fit();
    q.bank.clear();
    q.bank.shrink_to_fit();
    q.state = REQ_ACTIVE;
    return MING_OK;
}

// Reads the flags of the step queued in slot `sl` and retires the rows that
// finished by then: their results stay on the device until fetched, their
// sequences release their pages, and the last active rows move into their
// places (queued behind every step already on the stream).
int retire(ming_loop* lp, int sl) {
    if (!lp->pending[sl]) return MING_OK;
    ming_ctx* c = lp->c;
    CK(cudaEventSynchronize(lp->ev[sl]));
    lp->pending[sl] = false;
    const std::vector<int>& at = lp->rows_at[sl];
    const int* done = lp->h_flags + (size_t)sl * (2 * lp->R + 1);
    const int* nout = done + lp->R;
    if (done[2 * lp->R]) return check_dev_err(c);  // a bounded device wait of that step gave up
    std::vector<int> fin;
    for (int row = 0; row < (int)at.size(); row++) {
        auto it = lp->reqs.find(at[row]);
        if (it == lp->reqs.end()) continue;
        Request& q = it->second;
        if (q.state != REQ_ACTIVE || !done[row]) continue;
        q.n_out = nout[row];
        q.state = REQ_DONE;
        fin.push_back(at[row]);
    }
    if (fin.empty()) return MING_OK;
    std::vector<int> pairs;
    for (int id : fin) {
        const int row = (int)(std::find(lp->rows.begin(), lp->rows.end(), id) - lp->rows.begin());
        const int last = (int)lp->rows.size() - 1;
        if (row != last) {
            pairs.push_back(row);
            pairs.push_back(last);
            lp->rows[row] = lp->rows[last];
        }
        lp->rows.pop_back();
        int rc = seq_release(c, lp->reqs[id].seq);
        if (rc) return rc;
        lp->reqs[id].seq = -1;
    }
    if (!pairs.empty()) {
        // pairs are applied in order: a later pair may move a row an earlier
        // pair filled, which the kernel's sequential loop respects
        CK(cudaMemcpyAsync(lp->d_pairs, pairs.data(), pairs.size() * 4, cudaMemcpyHostToDevice, c->stream));
        loop_move_kernel<<<1, 256, 0, c->stream>>>(lp->d, lp->d_pairs, (int)pairs.size() / 2, lp->H, lp->LAT);
        CK(cudaGetLastError());
    }
    return MING_OK;
}

int fill_rows(ming_loop* lp) {
    while (!lp->queue.empty() && (int)lp->rows.size() < lp->R) {
        const int id = lp->queue.front();
        const int row = (int)lp->rows.size();
        int rc = admit(lp, id, row);
        if (rc == MING_ERR_NOMEM && !lp->rows.empty()) return MING_OK;  // pages free up as rows retire
        lp->queue.pop_front();
        if (rc) {
            Request& q = lp->reqs[id];
            q.state = REQ_DONE;
            q.error = ming_cuda_last_error();
            q.n_out = 0;
            return rc;
        }
        lp->rows.push_back(id);
    }
    return MING_OK;
}

}  // namespace

extern "C" {

void ming_cuda_default_sample_params(ming_sample_params* p) {
    if (!p) return;
    p->max_steps = 1000;
    p->max_len = 512;
    p->cfg = 2.0f;
    p->sigma = 0.25f;
    p->temperature = 0.0f;
}

int ming_cuda_loop_create(ming_ctx* c, int max_rows, const ming_sample_params* p, ming_loop** out) {
    if (!c || !c->finalized || !p || !out) return fail(MING_ERR_INVALID, "bad argument");
    const ming_cfg& f = c->cfg;
    if (f.layers < 1 || f.dit_mode == MING_DIT_NONE) return fail(MING_ERR_INVALID, "the loop needs the LM and the flow head");
    if (!c->agg_proj_on && c->agg.empty()) return fail(MING_ERR_INVALID, "the loop needs an aggregator");
    if (f.dit_cond_dim != f.hidden) return fail(MING_ERR_INVALID, "the flow head's condition must be the LM hidden state");
    if (max_rows < 1 || max_rows > std::min({f.max_batch, f.dit_max_batch, f.max_seqs}))
        return fail(MING_ERR_INVALID, "max_rows exceeds max_batch, dit_max_batch or max_seqs");
    if (p->max_steps < 1 || p->max_len < 2) return fail(MING_ERR_INVALID, "bad sampling limits");
    if (!(p->temperature >= 0.f) || !(p->sigma >= 0.f)) return fail(MING_ERR_INVALID, "sigma and temperature must be >= 0");
    CK(cudaSetDevice(c->device));
    std::unique_ptr<ming_loop> lp(new ming_loop());
    lp->c = c;
    lp->R = max_rows;
    lp->H = f.hidden;
    lp->LAT = f.dit_latent;
    lp->FL = f.dit_frames * f.dit_latent;
    lp->token = f.dit_mode == MING_DIT_TOKEN;
    lp->p = *p;
    lp->shift = p->sigma * std::sqrt(p->temperature);  // cfmSampleRaw's shift_k
    lp->sde = lp->shift != 0.f;
    lp->cap = std::min(p->max_len, f.max_ctx - 2);
    const int R = max_rows, H = lp->H, LAT = lp->LAT;
    // one allocation for every per-row array, each 256-byte aligned
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 255) / 256 * 256;
        return o;
    };
    const size_t o_z = take((size_t)R * H * 2), o_stop = take(R * 4), o_hist = take((size_t)R * LAT * 2),
                 o_step = take(R * 4), o_budget = take(R * 4), o_done = take(R * 4), o_nout = take(R * 4),
                 o_seed = take(R * 8), o_bank = take(R * sizeof(void*)), o_lat = take(R * sizeof(void*)),
                 o_oz = take(R * sizeof(void*)), o_os = take(R * sizeof(void*)), o_pairs = take((size_t)2 * R * 4);
    CK(cudaMalloc(&lp->d_block, off));
    CK(cudaMemset(lp->d_block, 0, off));
    uint8_t* base = static_cast<uint8_t*>(lp->d_block);
    LoopRows& r = lp->d;
    r.z = reinterpret_cast<uint16_t*>(base + o_z);
    r.stop = reinterpret_cast<float*>(base + o_stop);
    r.hist = reinterpret_cast<uint16_t*>(base + o_hist);
    r.step = reinterpret_cast<int*>(base + o_step);
    r.budget = reinterpret_cast<int*>(base + o_budget);
    r.done = reinterpret_cast<int*>(base + o_done);
    r.n_out = reinterpret_cast<int*>(base + o_nout);
    r.seed = reinterpret_cast<unsigned long long*>(base + o_seed);
    r.bank = reinterpret_cast<const uint16_t**>(base + o_bank);
    r.out_lat = reinterpret_cast<uint16_t**>(base + o_lat);
    r.out_z = reinterpret_cast<uint16_t**>(base + o_oz);
    r.out_stop = reinterpret_cast<float**>(base + o_os);
    lp->d_pairs = reinterpret_cast<int*>(base + o_pairs);
    CK(cudaHostAlloc(reinterpret_cast<void**>(&lp->h_flags), (size_t)2 * (2 * R + 1) * 4, cudaHostAllocDefault));
    for (cudaEvent_t& e : lp->ev) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    *out = lp.release();
    return MING_OK;
}

int ming_cuda_loop_submit(ming_loop* lp, const uint16_t* embeds, int L, const uint16_t* prompt_latent,
                          const uint16_t* noise_bank, int bank_steps, uint64_t seed, int want_trace, int* req) {
    if (!lp || !embeds || !req) return fail(MING_ERR_INVALID, "null argument");
    if (L < 1) return fail(MING_ERR_INVALID, "empty prompt");
    if (L >= lp->cap) return fail(MING_ERR_INVALID, "prompt too long: no step fits under max_len");
    if (noise_bank && bank_steps < 1) return fail(MING_ERR_INVALID, "empty noise bank");
    Request q;
    q.L = L;
    q.budget = std::min(lp->p.max_steps, lp->cap - L);
    if (noise_bank) q.budget = std::min(q.budget, bank_steps);
    q.embeds.assign(embeds, embeds + (size_t)L * lp->H);
    q.hist0.assign(lp->LAT, 0);
    if (prompt_latent && lp->token) q.hist0.assign(prompt_latent, prompt_latent + lp->LAT);
    if (noise_bank) q.bank.assign(noise_bank, noise_bank + (size_t)q.budget * (LOOP_STEPS + 1) * lp->FL);
    q.seed = seed;
    q.trace = want_trace != 0;
    const int id = lp->next_id++;
    lp->reqs[id] = std::move(q);
    lp->queue.push_back(id);
    *req = id;
    CK(cudaSetDevice(lp->c->device));
    return fill_rows(lp);
}

int ming_cuda_loop_step(ming_loop* lp, int* active, int* queued) {
    if (!lp) return fail(MING_ERR_INVALID, "null loop");
    ming_ctx* c = lp->c;
    CK(cudaSetDevice(c->device));
    int rc;
    const int sl = (int)(lp->nstep & 1), prev = sl ^ 1;
    if (!lp->rows.empty()) {
        const int B = (int)lp->rows.size();
        std::vector<int> ids(B);
        for (int i = 0; i < B; i++) ids[i] = lp->reqs[lp->rows[i]].seq;
        if ((rc = prepare_rows(c, B, ids.data(), 1))) return rc;
        if (!c->cells_null) {
            // per-step output cells of the decode kernels stay null in the loop
            static uint16_t* const null_out = nullptr;
            static float* const null_stop = nullptr;
            CK(cudaMemcpyAsync(c->out_cell, &null_out, sizeof(void*), cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(c->stop_cell, &null_stop, sizeof(void*), cudaMemcpyHostToDevice, c->stream));
            c->cells_null = true;
        }
        cudaGraphExec_t g;
        if ((rc = loop_graph(lp, B, &g))) return rc;
        // the slot's flags are free: the step that last used it was retired
        if ((rc = retire(lp, sl))) return rc;
        CK(cudaGraphLaunch(g, c->stream));
        for (int i = 0; i < B; i++) c->seqs[ids[i]].len += 1;
        // the rows' flags and the device error flag travel back behind the step
        int* hf = lp->h_flags + (size_t)sl * (2 * lp->R + 1);
        CK(cudaMemcpyAsync(hf, lp->d.done, (size_t)B * 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaMemcpyAsync(hf + lp->R, lp->d.n_out, (size_t)B * 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaMemcpyAsync(hf + 2 * lp->R, c->dev_err, 4, cudaMemcpyDeviceToHost, c->stream));
        CK(cudaEventRecord(lp->ev[sl], c->stream));
        lp->rows_at[sl] = lp->rows;
        lp->pending[sl] = true;
        lp->nstep++;
    }
    // the previous step's flags (this step is already queued behind it)
    if ((rc = retire(lp, prev))) return rc;
    if (lp->rows.empty() && lp->pending[sl]) {
        if ((rc = retire(lp, sl))) return rc;
    }
    if ((rc = fill_rows(lp))) return rc;
    if (active) *active = (int)lp->rows.size();
    if (queued) *queued = (int)lp->queue.size();
    return MING_OK;
}

int ming_cuda_loop_result(ming_loop* lp, int req, uint16_t* latents, int cap, int* n, uint16_t* z_trace, float* stop_trace) {
    if (!lp || !n) return fail(MING_ERR_INVALID, "null argument");
    auto it = lp->reqs.find(req);
    if (it == lp->reqs.end()) return fail(MING_ERR_INVALID, "unknown request");
    Request& q = it->second;
    if (q.state != REQ_DONE) {
        *n = -1;
        return MING_OK;
    }
    if (!q.error.empty()) {
        const std::string e = q.error;
        lp->reqs.erase(it);
        return fail(MING_ERR_CUDA, "request failed at admission: " + e);
    }
    if (q.n_out > cap) return fail(MING_ERR_INVALID, "result buffer too small: " + std::to_string(q.n_out) + " latents");
    ming_ctx* c = lp->c;
    CK(cudaSetDevice(c->device));
    CK(cudaStreamSynchronize(c->stream));
    if (latents && q.n_out) CK(cudaMemcpy(latents, q.d_lat, (size_t)q.n_out * lp->FL * 2, cudaMemcpyDeviceToHost));
    if (stop_trace && q.n_out) CK(cudaMemcpy(stop_trace, q.d_stop, (size_t)q.n_out * 4, cudaMemcpyDeviceToHost));
    if (z_trace && q.n_out) {
        if (!q.d_z) return fail(MING_ERR_INVALID, "the request was submitted without a trace");
        CK(cudaMemcpy(z_trace, q.d_z, (size_t)q.n_out * lp->H * 2, cudaMemcpyDeviceToHost));
    }
    *n = q.n_out;
    q.free_device();
    lp->reqs.erase(it);
    return MING_OK;
}

int ming_cuda_loop_destroy(ming_loop* lp) {
    if (!lp) return MING_OK;
    cudaSetDevice(lp->c->device);
    cudaStreamSynchronize(lp->c->stream);
    for (auto& q : lp->reqs)
        if (q.second.seq >= 0) seq_release(lp->c, q.second.seq);
    cudaStreamSynchronize(lp->c->stream);
    delete lp;
    return MING_OK;
}

int ming_cuda_sample_latents(ming_ctx* c, const uint16_t* embeds, int L, const uint16_t* prompt_latent,
                             const ming_sample_params* p, const uint16_t* noise_bank, int bank_steps, uint64_t seed,
                             uint16_t* latents, int cap, int* n, uint16_t* z_trace, float* stop_trace) {
    if (!n) return fail(MING_ERR_INVALID, "null argument");
    ming_sample_params dp;
    ming_cuda_default_sample_params(&dp);
    ming_loop* lp = nullptr;
    int rc = ming_cuda_loop_create(c, 1, p ? p : &dp, &lp);
    if (rc) return rc;
    int id = -1;
    rc = ming_cuda_loop_submit(lp, embeds, L, prompt_latent, noise_bank, bank_steps, seed, z_trace != nullptr, &id);
    int active = 1;
    while (!rc && active) rc = ming_cuda_loop_step(lp, &active, nullptr);
    if (!rc) rc = ming_cuda_loop_result(lp, id, latents, cap, n, z_trace, stop_trace);
    const std::string err = rc ? ming_cuda_last_error() : "";
    ming_cuda_loop_destroy(lp);
    if (rc) return fail(rc, err);
    return MING_OK;
}

}  // extern "C"
