/*
 * ming_cuda.h — C ABI of the B200 (sm_100a) implementation of ming-tts-serve's
 * per-step hot path: the KV-cached Qwen2 LM decode step and the DiT
 * flow-matching head.
 *
 * Plain C types only (bf16 values travel as uint16_t bit patterns). Every call
 * returns MING_OK (0) or an error code; ming_cuda_last_error() gives the
 * message of the calling thread's last failure. This mirrors mlx-c's
 * convention that the reference binds (src/mlx.zig:8-17, `check()` at
 * src/mlx.zig:431): an int status plus out-pointers.
 *
 * Threading: one context per GPU; calls on one context come from one thread
 * (the reference runs all GPU work on one engine thread,
 * src/ming_service.zig:11-14). Work is queued on the context's stream;
 * calls that return data to host memory synchronise that stream.
 *
 * Pointer kinds: functions taking `ptr_kind` accept host pointers
 * (MING_PTR_HOST, copied through the context's staging buffers) or device
 * pointers on the context's GPU (MING_PTR_DEVICE, no copies, asynchronous).
 */
#ifndef MING_CUDA_H
#define MING_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MING_OK 0
#define MING_ERR_INVALID 1  /* bad argument, shape or state */
#define MING_ERR_CUDA 2     /* a CUDA call failed */
#define MING_ERR_NOMEM 3    /* device memory or KV pages exhausted */
#define MING_ERR_MISSING 4  /* a required weight was not loaded */

enum { MING_DTYPE_BF16 = 0, MING_DTYPE_F32 = 1, MING_DTYPE_U32 = 2 };
enum { MING_PTR_HOST = 0, MING_PTR_DEVICE = 1 };
enum { MING_DIT_NONE = 0, MING_DIT_TOKEN = 1, MING_DIT_ADALN = 2 };

typedef struct ming_ctx ming_ctx;

/* Model and runtime shape. ming_cuda_default_cfg() fills the Qwen2-0.5B LM of
 * Ming-3.0-tts (src/ming_model.zig:37-53,500-504) with the reference's
 * token-conditioned flow head (8 blocks x 1024) and aggregator. */
typedef struct ming_cfg {
    /* LM */
    int hidden, layers, heads, kv_heads, head_dim, ff;
    float rope_theta, rms_eps;
    int weight_bits; /* 16 (bf16), 8 or 4 (MLX affine, group_size) */
    int group_size;
    /* KV cache and batching */
    int page_size;    /* positions per page; must be 16 */
    int max_seqs;     /* sequences alive at once */
    int max_pages;    /* pages in the pool */
    int max_ctx;      /* positions per sequence */
    int max_batch;    /* rows per decode step */
    int max_prefill;  /* rows per prefill chunk */
    /* flow head */
    int dit_mode; /* MING_DIT_NONE / TOKEN / ADALN */
    int dit_hidden, dit_blocks, dit_heads, dit_ff, dit_latent, dit_frames, dit_cond_dim, dit_freq_dim;
    int dit_max_batch;
    /* aggregator (token mode only; 0 blocks = none) */
    int agg_blocks;
    /* VAE decoder (audio.decoder.*; 0 layers = none, the reference's is 24):
     * Qwen2 layers of the LM's width with a causal sliding window, latents
     * upsampled x4, an ISTFT head (n_fft 3528, hop 882) */
    int vae_layers, vae_ff, vae_window;
    int vae_max_latents; /* latents per ming_cuda_vae_decode call */
} ming_cfg;

void ming_cuda_default_cfg(ming_cfg* cfg);

/* Replaces Model.load's device side (src/ming_model.zig:923): creates the
 * context on `device`. Weights follow with ming_cuda_load_tensor. */
int ming_cuda_create(int device, const ming_cfg* cfg, ming_ctx** out);

/* One tensor of model.safetensors under the reference's names
 * (src/ming_model.zig:546-561,728-741,938-965), e.g.
 * "model.model.layers.3.self_attn.q_proj.weight". Quantized linears come as
 * "<prefix>.weight" (U32, [out, in*bits/32]) + ".scales" + ".biases" (BF16,
 * [out, in/group]), MLX's QuantizedLinear layout. The data is copied. */
int ming_cuda_load_tensor(ming_ctx* ctx, const char* name, int dtype, const int64_t* shape, int ndim, const void* host);

/* Model.load's file side (src/ming_model.zig:316-350,923-1005): reads a
 * safetensors checkpoint (`path` a file, or a directory holding
 * model.safetensors) and loads the tensors this library runs (names under
 * model.model., stop_head, flowloss., linear_proj_audio, adaln_head,
 * aggregator., audio.decoder.) with ming_cuda_load_tensor: BF16 and U32 as stored, F32 and
 * F16 rounded to bf16 (the reference casts to its bf16 model dtype) except
 * rotary inv_freq buffers, which stay F32; other names and dtypes are
 * skipped. *n_loaded (may be NULL) = tensors loaded. With ctx NULL the file
 * is only validated (no GPU needed). */
int ming_cuda_load_safetensors(ming_ctx* ctx, const char* path, int* n_loaded);

/* Checks that every weight is present, repacks them into the kernels' tile
 * layout on the device, precomputes the flow schedule tables, frees the
 * staged copies. Must precede any compute call. */
int ming_cuda_finalize(ming_ctx* ctx);

/* Sequences own KV pages (KvCache.init/deinit, src/ming_model.zig:638-662). */
int ming_cuda_seq_alloc(ming_ctx* ctx, int* seq_id);
int ming_cuda_seq_free(ming_ctx* ctx, int seq_id);
int ming_cuda_seq_len(ming_ctx* ctx, int seq_id, int* len);
/* Truncates a sequence to `len` positions (pages are kept for reuse). */
int ming_cuda_seq_truncate(ming_ctx* ctx, int seq_id, int len);

/* Model.lmForward for a multi-row prompt (QStack.forward with L > 1,
 * src/ming_model.zig:566-614): x [L][hidden] at positions len..len+L-1,
 * appends K/V. out [L][hidden] post-norm hidden (may be NULL), stop [L]
 * p(stop) of each row (may be NULL). */
int ming_cuda_lm_prefill(ming_ctx* ctx, int seq_id, const uint16_t* x, int L, uint16_t* out, float* stop, int ptr_kind);

/* One decode step for B sequences (QStack.forward decode branch ->
 * decodeFused -> fused.lmLayer x 24, src/ming_model.zig:529-544,566-575,
 * src/ming_fused.zig:597-614; stopProb src/ming_model.zig:1033-1038):
 * x [B][hidden] -> out [B][hidden], stop [B]. Runs one captured CUDA graph. */
int ming_cuda_lm_decode(ming_ctx* ctx, int B, const int* seq_ids, const uint16_t* x, uint16_t* out, float* stop,
                        int ptr_kind);

/* `steps` decode steps feeding each step's output hidden state back as the
 * next input (the benchmark's LM token loop): out [steps][B][hidden],
 * stop [steps][B] (either may be NULL). */
int ming_cuda_lm_generate(ming_ctx* ctx, int B, const int* seq_ids, const uint16_t* x0, int steps, uint16_t* out,
                          float* stop, int ptr_kind);

/* ming_cuda_lm_decode for callers that cannot allocate device memory during a
 * step: a host real-time audio thread must not block in cudaMalloc, and a
 * process whose device memory is budgeted by another runtime has cudaMalloc
 * refused once the budget is spent. Same arguments and results as
 * ming_cuda_lm_decode (within bf16 rounding); it instantiates no CUDA graph
 * and keeps its one scratch buffer, the split-K attention partials, in a
 * fixed 4 MiB array compiled into the library (held by every GPU that loads
 * the library until the process exits). A step needing more than that
 * (B x ceil(max_ctx / 256) x heads x 264 bytes) is rejected with
 * MING_ERR_INVALID. The first call on a device looks up the array's device
 * address; make that first call before any stream capture. All calls on a
 * device share the array and its contents persist between calls; nothing in
 * it needs to start at zero, but calls that overlap on the GPU (other
 * streams, other contexts on the same device) race on it. At most 16 query
 * heads. With host pointers a bounded device wait that gave up is reported
 * by this call (MING_ERR_CUDA); with device pointers, by the next
 * ming_cuda_sync.
 * No reference counterpart: the reference's MLX allocator owns all memory. */
int ming_cuda_lm_decode_noalloc(ming_ctx* ctx, int B, const int* seq_ids, const uint16_t* x, uint16_t* out, float* stop,
                                int ptr_kind);

/* Model.cfmSample (src/ming_model.zig:1143-1215): 10 Euler steps with CFG.
 * Token mode: z [B][cond_dim], hist [B][latent], noise [B][latent],
 * sde [10][B][latent] or NULL. adaLN mode: hist unused, noise/y
 * [B][frames][latent], sde [10][B][frames][latent] or NULL.
 * shift = sigma * sqrt(temperature) (0 disables the SDE term). */
int ming_cuda_cfm_sample(ming_ctx* ctx, int B, const uint16_t* z, const uint16_t* hist, const uint16_t* noise,
                         const uint16_t* sde, float cfg, float shift, uint16_t* y, int ptr_kind);

/* The same Euler update restricted to steps [step0, step0+nsteps) starting
 * from latent y_in (layout of `noise`); cfm_sample is steps [0, 10) from the
 * noise. Lets a caller replay the sampler one step at a time (the reference's
 * teacher-forced parity method, src/ming_parity.zig:6-8). */
int ming_cuda_cfm_steps(ming_ctx* ctx, int B, const uint16_t* z, const uint16_t* hist, const uint16_t* y_in,
                        const uint16_t* sde, float cfg, float shift, int step0, int nsteps, uint16_t* y, int ptr_kind);

/* Model.aggregate (src/ming_model.zig:1040-1053,1153-1157): latent [B][latent]
 * -> next LM input rows [B][hidden]. */
int ming_cuda_aggregate(ming_ctx* ctx, int B, const uint16_t* latent, uint16_t* out, int ptr_kind);

/* ---- the autoregressive loop: sampleLatents and a request scheduler ---- */

/* SampleParams (src/ming_model.zig:1368-1373) plus the position cap the
 * reference fixes at MAX_CACHE_LEN (src/ming_model.zig:46-47). */
typedef struct ming_sample_params {
    int max_steps;     /* latents per request at most (1000) */
    int max_len;       /* prompt + generated positions (512) */
    float cfg;         /* classifier-free guidance scale (2.0) */
    float sigma;       /* SDE scale (0.25) */
    float temperature; /* SDE temperature (0.0: shift = sigma * sqrt(temperature) = 0, no SDE term) */
} ming_sample_params;

void ming_cuda_default_sample_params(ming_sample_params* p);

/* sampleLatents (src/ming_model.zig:1388-1480) for one sequence, on the
 * device: prefill `embeds` [L][hidden]; then per step the flow head on the
 * last hidden state z (cfmSample, with the previous latent as history in
 * token mode; prompt_latent [latent] seeds it, NULL = zeros), the aggregator,
 * one LM step, and the stop rule on z's stop probability: the step's latent
 * is emitted, then the loop ends if p > 0.5 and step > 3, or after
 * min(max_steps, max_len - L) steps. Noise: the reference's replay bank
 * noise_bank [bank_steps][11][frames * latent] (row 0 the start noise, rows
 * 1..10 the SDE draws; at most bank_steps steps), or, with noise_bank NULL,
 * the library's seeded stream (SplitMix64 + Box-Muller over
 * (seed, "loop.noise.<step>"), 11 rows per step). Host pointers. latents
 * [cap][frames * latent], *n = latents emitted; z_trace [cap][hidden] and
 * stop_trace [cap] (either may be NULL) receive each step's z and p(stop),
 * the reference's Trace (src/ming_model.zig:1376-1385). */
int ming_cuda_sample_latents(ming_ctx* ctx, const uint16_t* embeds, int L, const uint16_t* prompt_latent,
                             const ming_sample_params* p, const uint16_t* noise_bank, int bank_steps, uint64_t seed,
                             uint16_t* latents, int cap, int* n, uint16_t* z_trace, float* stop_trace);

/* The same loop over up to max_rows concurrent requests (continuous
 * batching in place of the reference's one-at-a-time FIFO,
 * src/ming_service.zig:175-206,277-287). One CUDA graph per row count runs a
 * whole step for every active row; stop flags come back one step behind
 * (the next step is already queued); finished rows retire and queued
 * requests take their places, their prompts prefilling between two steps.
 * The context must not run other work while a loop has active rows (the
 * loop uses its step buffers). */
typedef struct ming_loop ming_loop;
int ming_cuda_loop_create(ming_ctx* ctx, int max_rows, const ming_sample_params* p, ming_loop** out);
/* Queues one request (arguments as in ming_cuda_sample_latents; want_trace
 * keeps per-step z for loop_result) and admits it at once if a row is free. */
int ming_cuda_loop_submit(ming_loop* lp, const uint16_t* embeds, int L, const uint16_t* prompt_latent,
                          const uint16_t* noise_bank, int bank_steps, uint64_t seed, int want_trace, int* req);
/* Runs one step of every active row; *active and *queued (may be NULL)
 * report the rows still running and the requests waiting for a row. */
int ming_cuda_loop_step(ming_loop* lp, int* active, int* queued);
/* A finished request's latents [cap][frames * latent] and traces; *n = -1
 * while it is still queued or running. Fetching releases the request. */
int ming_cuda_loop_result(ming_loop* lp, int req, uint16_t* latents, int cap, int* n, uint16_t* z_trace, float* stop_trace);
int ming_cuda_loop_destroy(ming_loop* lp);

/* Model.vaeDecode (src/ming_model.zig:1257-1300): latents [T][64] (bf16) ->
 * waveform [T * 4 * 882] f32 at 44.1 kHz. fc1 (64 -> hidden), linear upsample
 * x4 in f32 (linearUpsample, :1303-1342), the decoder's Qwen2 layers in f32
 * activations with a causal sliding window of vae_window positions
 * (QStack.forward with a window, :566-614, slidingMask :617-635), final norm,
 * the head linear (hidden -> 3530), then the ISTFT: magnitude
 * min(exp(m), 100) and phase of 1765 bins, irfft of 3528 points, the
 * checkpoint's window, overlap-add at hop 882, division by the window
 * envelope and the "same" trim of 1323 samples per side. */
int ming_cuda_vae_decode(ming_ctx* ctx, const uint16_t* latents, int T, float* wave, int ptr_kind);

/* The context's CUDA stream (a cudaStream_t), for event timing by callers. */
int ming_cuda_get_stream(ming_ctx* ctx, void** stream);
int ming_cuda_sync(ming_ctx* ctx);
/* Kernels one decode step of B rows launches: 1 when the persistent decode
 * kernel serves B (B <= 4 and a device that co-schedules one block per SM),
 * else the per-kernel path's count. No reference counterpart: the reference
 * dispatches its Metal kernels itself and exposes no such count. */
int ming_cuda_step_kernels(ming_ctx* ctx, int B, int* n);
int ming_cuda_destroy(ming_ctx* ctx);
const char* ming_cuda_last_error(void);

/* ---- inspection (tests) ---- */
/* Reads positions [pos0, pos0+n) of one layer's cache through the block
 * table: k, v host [kv_heads][n][head_dim] bf16. */
int ming_cuda_kv_read(ming_ctx* ctx, int seq_id, int layer, int pos0, int n, uint16_t* k, uint16_t* v);
/* Writes positions [pos0, pos0+n) of one layer's cache through the block
 * table (k, v host [kv_heads][n][head_dim] bf16), allocating pages as needed;
 * pos0 <= the sequence's length, which grows to pos0 + n if shorter. The
 * device side indexes the pool with the same function the decode kernels
 * append with, so a write followed by ming_cuda_kv_read round-trips bit for
 * bit. Restores a saved prompt cache; tests inject known caches with it.
 * No reference counterpart (the reference's KvCache holds MLX arrays,
 * src/ming_model.zig:638-662). */
int ming_cuda_kv_write(ming_ctx* ctx, int seq_id, int layer, int pos0, int n, const uint16_t* k, const uint16_t* v);
/* Dequantizes a loaded linear back from its device tiles (the kernels' own
 * unpack path): out host [out][in] f32 in the reference's row order. */
int ming_cuda_unpack_linear(ming_ctx* ctx, const char* weight_name, float* out);
/* Timestep embeddings [10][dit_hidden] bf16 the flow head uses (host). */
int ming_cuda_flow_temb(ming_ctx* ctx, uint16_t* te);

#ifdef __cplusplus
}
#endif
#endif
