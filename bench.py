"""Benchmark of the B200 hot path (one JSON line on stdout from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]

Workload (default): the Ming LM token loop with
MLX-style affine 4-bit g64 weights, batch 1, a 128-token prefill, then decode
steps feeding each step's output hidden state back as the next input. A
"step" is one decode step of the batch (one token per sequence). Other
configs: 1 (bf16 LM, batch 1), 3 (4-bit, batch 32, ragged prompts),
4 (adaLN DiT head, one CFM sample of 10 Euler steps per step), 5 (the LM+DiT
loop), 6 (the VAE decoder, one 128-latent fragment per step).

value  : device-timed throughput with inputs resident in HBM (CUDA events on
         the library's stream around exactly K steps, max over ranks).
e2e    : the same metric through the public C ABI call a user makes
         (ming_cuda_lm_decode with pinned host buffers: each step copies its
         input in and reads its hidden state + stop probability back).
--impl reference: the reference's CPU path restated (the oracle port,
         OpenMP on the host cores) on the same workload; rank 0 only.

Multi-GPU (torchrun): one independent replica per GPU (the path does not
shard); value is the sum over replicas of tokens / the max time over ranks.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ming-tts-serve_b200"))

METRIC = "LM decode tokens/s (batch 1 & 32) per B200 and at 1/2/4/8 GPUs; % HBM roofline"

CONFIGS = {
    1: dict(name="LM token loop, bf16, batch 1, 64-token prefill + 256 decode steps (BASELINE configs[0])",
            bits=16, batch=1, prefill=64, decode=256, seed=0),
    2: dict(name="LM token loop, MLX affine 4-bit g64, batch 1, 128-token prefill + 1024 decode steps (BASELINE configs[1])",
            bits=4, batch=1, prefill=128, decode=1024, seed=0),
    3: dict(name="LM batched decode, 4-bit g64, 32 sequences, prompts U[32,512], 512 decode steps, 16-token pages (BASELINE configs[2])",
            bits=4, batch=32, prefill=None, decode=512, seed=0),
    4: dict(name="DiT adaLN flow head, 6x768, 4x64 latent patch, 10 Euler steps, CFG, batch 1 (BASELINE configs[3])",
            dit=True, batch=1, seed=1),
    41: dict(name="DiT adaLN flow head, 6x768, 4x64 latent patch, 10 Euler steps, CFG, batch 32 (BASELINE configs[3])",
             dit=True, batch=32, seed=1),
    5: dict(name="LM+DiT loop: 4-bit LM batch 64, 2048-token prefill, then per step an LM decode step, the adaLN head "
                 "(10 Euler steps, CFG) and the latent's 64->896 projection into the next LM input (BASELINE configs[4])",
            bits=4, batch=64, prefill=2048, seed=0, loop=True),
    6: dict(name="VAE decoder (Model.vaeDecode): one fragment of 128 latents [128][64] -> 44.1 kHz waveform of "
                 "128 x 4 x 882 samples (10.24 s): fc1, x4 upsample, 24 Qwen2 layers (896, ff 4864, sliding window 64, "
                 "f32 activations, bf16 weights), final norm, ISTFT head",
            vae=True, latents=128, seed=2),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """Samples nvidia-smi during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = max(smax, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        import torch.distributed as dist
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    return ws, rank, local


def dist_max(x, ws):
    """Max of a per-rank scalar over all ranks (device time is the max over ranks)."""
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_throughput(local_ms, rows_per_rank, steps, ws):
    """Whole-job throughput of independent replicas: every rank processed
    rows_per_rank * steps units; the job took the slowest rank's time."""
    ms = dist_max(local_ms, ws)
    return ws * rows_per_rank * steps / (ms / 1e3), ms


def profile_range(start):
    """BENCH_PROFILE_RANGE=1: bracket the timed region with cudaProfilerStart/Stop
    (for `ncu --profile-from-start off`, which then captures exactly its launches)."""
    if os.environ.get("BENCH_PROFILE_RANGE") != "1":
        return
    import torch
    torch.cuda.synchronize()
    (torch.cuda.profiler.start if start else torch.cuda.profiler.stop)()


def dist_barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def lm_workload(cfgid, local, steps, warmup, W=None):
    import ming_b200 as M
    from ming_b200 import synth
    c = CONFIGS[cfgid]
    B = c["batch"]
    if c["prefill"] is None:  # ragged prompts U[32, 512]
        rng = np.random.default_rng(c["seed"])
        lens = rng.integers(32, 513, size=B).tolist()
    else:
        lens = [c["prefill"]] * B
    max_ctx = ((max(lens) + warmup + steps + 2 + 255) // 256) * 256
    pages = sum((L + warmup + steps + 2 + 15) // 16 for L in lens) + 16
    t0 = time.time()
    if W is None:
        W = synth.lm_weights(seed=c["seed"], bits=c["bits"], layers=24)
        log(f"[bench] weights generated in {time.time() - t0:.1f}s ({synth.nbytes(W) / 1e6:.1f} MB)")
    # a prompt prefills in one chunk (up to 2048 rows: the tcgen05 linear's row blocks)
    cfg = M.default_cfg(weight_bits=c["bits"], dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=max_ctx, max_pages=pages,
                        max_batch=max(B, 1), max_seqs=max(B, 1), max_prefill=max(512, min(2048, max(lens))))
    ctx = M.Context(cfg, device=local, weights=W)
    seqs = []
    last = []
    for b, L in enumerate(lens):
        s = ctx.seq_alloc()
        x = synth.normal_bf16(c["seed"], f"bench.prompt.{b}", (L, 896))
        out, _ = ctx.prefill(s, x)
        seqs.append(s)
        last.append(out[-1])
    return ctx, seqs, lens, np.stack(last), W


def algorithmic_bytes_lm(W, lens_now, B):
    """Bytes a decode step must move: every weight once, the KV cache of
    every sequence (K and V, all layers) once, activations negligible."""
    w = sum(v.nbytes for k, v in W.items() if k.startswith("model.model.layers.")) + W["model.model.norm.weight"].nbytes \
        + W["stop_head.weight"].nbytes
    kv = sum(12288 * (L + 1) for L in lens_now)  # 24 layers x (K+V) x 2 heads x 64 x 2 B per position
    return w, kv


def run_ours(args, ws, rank, local):
    import torch

    cfgid = args.config
    c = CONFIGS[cfgid]
    torch.cuda.set_device(local)
    if c.get("dit"):
        return run_dit(args, ws, rank, local)
    if c.get("loop"):
        return run_loop(args, ws, rank, local)
    if c.get("vae"):
        return run_vae(args, ws, rank, local)
    res, W = measure_lm(cfgid, args, ws, rank, local, cpu=rank == 0 and ws == 1 and not args.no_cpu_baseline)
    if cfgid == 2 and not args.no_batch32:
        # the metric's second batch size: config 3 (32 sequences, ragged prompts) on the same weights,
        # timed over at most its own length (warm-up + timed steps within its 512 decode steps)
        import copy
        a3 = copy.copy(args)
        a3.steps = max(1, min(args.steps, CONFIGS[3]["decode"] - args.warmup))
        b32, _ = measure_lm(3, a3, ws, rank, local, cpu=False, W=W)
        res["batch32"] = {k: b32[k] for k in ("value", "unit", "ms_per_step", "steps", "warmup", "roofline", "e2e",
                                              "gpu_launches", "clocks")}
        res["batch32"]["config"] = b32["config"]
    return res


def measure_lm(cfgid, args, ws, rank, local, cpu, W=None):
    """One LM decode workload (configs 1-3): device-timed generate over K
    steps, then the same K steps through ming_cuda_lm_decode from pinned host
    buffers. Returns (JSON dict, weights)."""
    import torch

    import ming_b200 as M
    c = CONFIGS[cfgid]
    ctx, seqs, lens, x_last, W = lm_workload(cfgid, local, args.steps, args.warmup, W)
    B = len(seqs)
    stream = torch.cuda.ExternalStream(ctx.stream, device=local)
    xdev = torch.from_numpy(x_last.view(np.int16).copy()).to(f"cuda:{local}")
    nmax = max(args.steps, args.warmup)
    outdev = torch.empty((nmax, B, 896), dtype=torch.int16, device=f"cuda:{local}")
    stopdev = torch.empty((nmax, B), dtype=torch.float32, device=f"cuda:{local}")
    # warm-up (graph capture happens here)
    ctx.generate(seqs, xdev, args.warmup, kind=M.PTR_DEVICE, out=outdev, stop=stopdev)
    ctx.sync()
    lens_start = [ctx.seq_len(s) for s in seqs]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    dist_barrier(ws)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    profile_range(True)
    ev0.record(stream)
    ctx.generate(seqs, xdev, args.steps, kind=M.PTR_DEVICE, out=outdev, stop=stopdev)
    ev1.record(stream)
    ev1.synchronize()
    profile_range(False)
    torch.cuda.synchronize()
    dist_barrier(ws)
    ck = clocks.stop()
    ms_local = ev0.elapsed_time(ev1)
    value, ms = aggregate_throughput(ms_local, B, args.steps, ws)
    ms_step = ms / args.steps
    # roofline of the decode step (the captured graph): algorithmic bytes / step time
    wbytes, _ = algorithmic_bytes_lm(W, lens_start, B)
    kv_avg = sum(12288 * (L + args.steps / 2.0 + 1) for L in lens_start)
    step_bytes = wbytes + kv_avg
    hbm, tf, peak_kind = load_peaks()
    achieved = step_bytes / (ms_local / args.steps / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tp):
        traffic = json.load(open(tp)).get(f"config{cfgid}")
    # ---- e2e through the C ABI with pinned host buffers, one call per step ----
    xin = torch.from_numpy(x_last.view(np.int16).copy()).pin_memory()
    hout = torch.empty((B, 896), dtype=torch.int16).pin_memory()
    hstop = torch.empty((B,), dtype=torch.float32).pin_memory()
    for s, L in zip(seqs, lens_start):
        ctx.seq_truncate(s, L)
    ids = (M.ctypes.c_int * B)(*seqs)
    L_ = M.lib()
    # --e2e-api noalloc: the same loop through the allocation-free entry point
    dec = L_.ming_cuda_lm_decode_noalloc if args.e2e_api == "noalloc" else L_.ming_cuda_lm_decode
    for _ in range(min(args.warmup, 8)):
        M._check(dec(ctx._h, B, ids, M.ctypes.c_void_p(xin.data_ptr()), M.ctypes.c_void_p(hout.data_ptr()),
                     M.ctypes.c_void_p(hstop.data_ptr()), M.PTR_HOST))
    for s, L in zip(seqs, lens_start):
        ctx.seq_truncate(s, L)
    dist_barrier(ws)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        M._check(dec(ctx._h, B, ids, M.ctypes.c_void_p(xin.data_ptr()), M.ctypes.c_void_p(hout.data_ptr()),
                     M.ctypes.c_void_p(hstop.data_ptr()), M.PTR_HOST))
        xin.copy_(hout)  # feed the step's output back (host side, as a caller would)
    e2e_s = time.perf_counter() - t0
    e2e_s = dist_max(e2e_s, ws)
    e2e = {"value": ws * B * args.steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": B * 896 * 2,
           "d2h_bytes_per_step": B * 896 * 2 + B * 4,
           "api": ("ming_cuda_lm_decode_noalloc" if args.e2e_api == "noalloc" else "ming_cuda_lm_decode") + " (pinned host buffers)"}
    cpu = cpu_baseline(cfgid, W, lens, x_last, args.cpu_seconds) if cpu else None
    launches_per_step = ctx.step_kernels(B)
    kname = ("mega_kernel (persistent decode step, one launch)" if launches_per_step == 1 else
             "decode step (captured graph: %d kernels)" % launches_per_step)
    ctx.close()
    res = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 act / " + ("u4-g64" if c["bits"] == 4 else "u8-g64" if c["bits"] == 8 else "bf16") + " weights, f32 acc",
        "data": "synthetic (seeded random-init weights and N(0,1) embeddings, SplitMix64/Box-Muller)",
        "config": {"workload": c["name"], "batch_per_gpu": B, "prompt_lens": lens if len(lens) <= 4 else f"U[32,512] x{len(lens)}",
                   "kv_positions_at_start": lens_start if B <= 4 else [min(lens_start), max(lens_start)],
                   "kv_positions_timed": [min(lens_start), max(lens_start) + args.steps],
                   "timed_steps": f"{args.steps} decode steps after {args.warmup} warm-up steps (the workload's "
                                  f"{c['decode']} steps are its full length)",
                   "parallelism": f"replicas x{ws} (no collective)",
                   "l2": "inputs larger than L2: every step streams all weights (%.0f MB) from HBM" % (wbytes / 1e6)},
        "roofline": {"bound": "hbm", "kernel": kname,
                     "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_step": step_bytes, "traffic": traffic},
        "e2e": e2e, "gpu_launches": launches_per_step * args.steps, "clocks": ck, "cpu_baseline": cpu,
    }
    return res, W


def cpu_baseline(cfgid, W, lens, x_last, budget_s=20.0):
    """The oracle port (OpenMP, all host threads) on a bounded sample of the
    same workload: prefill (untimed) then decode steps until ~budget_s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from ming_b200 import synth
    O.set_threads(len(os.sched_getaffinity(0)))
    c = CONFIGS[cfgid]
    lm = O.Lm(W)
    B = len(lens)
    nb = min(B, 2)  # sequences sampled on the CPU
    caches, xs = [], []
    for b in range(nb):
        x = synth.normal_bf16(c["seed"], f"bench.prompt.{b}", (lens[b], 896))
        cch = lm.new_cache(lens[b] + 4096)
        out, _ = lm.forward(cch, x)
        caches.append(cch)
        xs.append(out[-1:])
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s and n < 1024:
        for b in range(nb):
            xs[b], _ = lm.forward(caches[b], xs[b])
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n * nb / dt, "unit": "tokens/s", "cores": O.threads(), "kind": "port",
            "sample": f"{n} decode steps x {nb} sequence(s) after an untimed {lens[0]}-token prefill, "
                      f"24 layers, same weights (CPU restatement, not MLX)"}


def run_dit(args, ws, rank, local):
    import torch

    import ming_b200 as M
    from ming_b200 import synth
    c = CONFIGS[args.config]
    B = c["batch"]
    W = synth.ada_weights(seed=c["seed"])
    cfg = M.default_cfg(layers=0, dit_mode=M.DIT_ADALN, dit_hidden=768, dit_blocks=6, dit_heads=12, dit_ff=3072,
                        dit_frames=4, dit_max_batch=max(B, 1), agg_blocks=0)
    ctx = M.Context(cfg, device=local, weights=W)
    z = synth.normal_bf16(c["seed"], "bench.dit.z", (B, 896))
    noise = synth.normal_bf16(c["seed"], "bench.dit.noise", (B, 4, 64))
    stream = torch.cuda.ExternalStream(ctx.stream, device=local)
    zd = torch.from_numpy(z.view(np.int16).copy()).cuda()
    nd = torch.from_numpy(noise.view(np.int16).copy()).cuda()
    yd = torch.empty_like(nd)
    L_ = M.lib()
    P = lambda t: M.ctypes.c_void_p(t.data_ptr())

    def step():
        M._check(L_.ming_cuda_cfm_sample(ctx._h, B, P(zd), None, P(nd), None, M.ctypes.c_float(2.0), M.ctypes.c_float(0.0),
                                         P(yd), M.PTR_DEVICE))

    for _ in range(args.warmup):
        step()
    ctx.sync()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    dist_barrier(ws)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    profile_range(True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    ev1.synchronize()
    profile_range(False)
    dist_barrier(ws)
    ck = clocks.stop()
    ms_local = ev0.elapsed_time(ev1)
    ms = dist_max(ms_local, ws)
    wbytes = synth.nbytes(W)
    hbm, tf, peak_kind = load_peaks()
    per_sample_bytes = 10 * wbytes  # weights once per Euler step
    # launches per cfm_sample call, mirroring the library's dispatch: a linear
    # of <= 64 rows is one kernel (the latent embedding's <= 8), larger ones two
    R, NC = 8 * B, 2 * B
    lin = lambda rows, small=64: 1 if rows <= small else 2
    launches = (lin(NC) + 10 + 7 * lin(10 * NC)
                + 10 * (lin(R, 8) + 6 * (4 * lin(R) + 1) + lin(R) + 1))
    achieved = per_sample_bytes / (ms_local / args.steps / 1e3) / 1e9
    hz = np.empty_like(noise)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        hz = ctx.cfm_sample(z, None, noise)
    e2e_s = dist_max(time.perf_counter() - t0, ws)
    ctx.close()
    return {"metric": "DiT flow-head CFM samples/s (10 Euler steps, CFG)", "value": ws * B * args.steps / (ms / 1e3),
            "unit": "samples/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random init)", "config": {"workload": c["name"], "batch_per_gpu": B},
            "roofline": {"bound": "hbm" if B < 16 else "tensor", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": peak_kind, "traffic": None},
            "e2e": {"value": ws * B * args.steps / e2e_s, "unit": "samples/s", "h2d_bytes_per_step": z.nbytes + noise.nbytes,
                    "d2h_bytes_per_step": noise.nbytes},
            "gpu_launches": launches * args.steps, "clocks": ck, "cpu_baseline": None}


def vae_workload(c):
    """The VAE decoder's weights (seeded random init of the real shapes) and one
    fragment's latents."""
    from ming_b200 import synth
    W = synth.vae_weights(seed=c["seed"])
    lat = synth.normal_bf16(c["seed"], "bench.vae.latents", (c["latents"], 64))
    return W, lat


def vae_work(W, T, window=64, heads=14):
    """Algorithmic FLOPs and bytes of one decode of T latents: the linears (fc1
    over T rows; the 24 layers and the head over F = 4T rows), the windowed
    attention (scores and P.V over min(i + 1, window) positions of row i), the
    weights read once, the latents in and the waveform out. The irfft (an FFT in
    the reference) is not counted."""
    F = 4 * T
    D = "audio.decoder"
    lin = lambda name: W[name + ".weight"].size
    layer_params = sum(v.size for k, v in W.items() if ".decoder.layers." in k and k.endswith("_proj.weight"))
    att = 4 * 64 * heads * sum(min(i + 1, window) for i in range(F)) * (layer_params > 0) * \
        sum(1 for k in W if k.endswith("self_attn.q_proj.weight"))
    flops = 2 * T * lin(D + ".fc1") + 2 * F * (layer_params + lin(D + ".head.out")) + att
    nbytes = sum(v.nbytes for v in W.values()) + T * 64 * 2 + F * 882 * 4
    return flops, nbytes


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        return max([i["num_threads"] for i in threadpool_info() if i.get("user_api") == "blas"] or [1])
    except ImportError:
        return len(os.sched_getaffinity(0))


def run_vae(args, ws, rank, local):
    """The VAE decoder (Model.vaeDecode) on one fragment of T latents per step:
    device-timed through ming_cuda_vae_decode on device buffers (CUDA events on
    the library's stream), e2e through the same call with pinned host buffers
    (the latents in, the waveform back). One replica per GPU. The CPU baseline
    is the oracle's f32 restatement (numpy, BLAS on the host cores)."""
    import torch

    import ming_b200 as M
    c = CONFIGS[args.config]
    T = c["latents"]
    t0 = time.time()
    W, lat = vae_workload(c)
    log(f"[bench] VAE weights generated in {time.time() - t0:.1f}s")
    cfg = M.default_cfg(layers=0, dit_mode=M.DIT_NONE, agg_blocks=0, vae_layers=24, vae_ff=4864, vae_window=64,
                        vae_max_latents=T)
    ctx = M.Context(cfg, device=local, weights=W)
    n_out = T * 4 * 882
    dev = f"cuda:{local}"
    stream = torch.cuda.ExternalStream(ctx.stream, device=local)
    ld = torch.from_numpy(lat.view(np.int16).copy()).to(dev)
    wd = torch.empty(n_out, dtype=torch.float32, device=dev)
    L_ = M.lib()
    P = lambda t: M.ctypes.c_void_p(t.data_ptr())

    def step(kind=M.PTR_DEVICE, src=ld, dst=wd):
        M._check(L_.ming_cuda_vae_decode(ctx._h, P(src), T, P(dst), kind))

    for _ in range(args.warmup):
        step()
    ctx.sync()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    dist_barrier(ws)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    profile_range(True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    ev1.synchronize()
    profile_range(False)
    dist_barrier(ws)
    ck = clocks.stop()
    ms_local = ev0.elapsed_time(ev1)
    value, ms = aggregate_throughput(ms_local, T, args.steps, ws)
    flops, nbytes = vae_work(W, T)
    hbm, tf, peak_kind = load_peaks()
    t_call = ms_local / args.steps / 1e3
    tensor_bound = flops / (tf * 1e12) >= nbytes / (hbm * 1e9)
    # e2e: pinned host latents in, pinned host waveform back, one call per step
    hl = torch.from_numpy(lat.view(np.int16).copy()).pin_memory()
    hw = torch.empty(n_out, dtype=torch.float32).pin_memory()
    for _ in range(min(args.warmup, 3)):
        step(M.PTR_HOST, hl, hw)
    dist_barrier(ws)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step(M.PTR_HOST, hl, hw)
    e2e_s = dist_max(time.perf_counter() - t0, ws)
    # launches per call, mirroring vae.cu and the linear dispatch: a linear over
    # more than 8 rows is a staging kernel and a tiled one (2 launches), up to 8
    # rows one; plus the upsample, 24 attention kernels, the spectrum and the
    # overlap-add kernels
    F = 4 * T
    lin = lambda rows: 1 if rows <= 8 else 2
    launches = lin(T) + 1 + 24 * (4 * lin(F) + 1) + lin(F) + 1 + lin(F) + 1
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        n, t0 = 0, time.perf_counter()
        while n < 1 or (time.perf_counter() - t0 < args.cpu_seconds and n < 8):
            O.vae_decode(W, lat, 24, window=64)
            n += 1
        dt = time.perf_counter() - t0
        cpu = {"value": n * T / dt, "unit": "latents/s", "cores": blas_threads(), "kind": "port",
               "sample": f"{n} decode(s) of the same {T} latents, 24 layers (the oracle's f32 numpy restatement, "
                         f"BLAS on the host cores; CPU restatement, not MLX)"}
    ctx.close()
    audio_s = T * 4 * 882 / 44100.0
    return {"metric": "VAE decode latents/s (one 128-latent fragment per call)", "value": value, "unit": "latents/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 activations as bf16 hi + lo parts, bf16 weights, f32 accumulation",
            "data": "synthetic (seeded random-init weights of the real shapes, N(0,1) latents)",
            "config": {"workload": c["name"], "latents_per_call": T, "rows_per_layer": F,
                       "audio_seconds_per_call": audio_s, "realtime_factor": (ms / args.steps / 1e3) / audio_s,
                       "parallelism": f"replicas x{ws} (no collective)",
                       "l2": "inputs larger than L2: every call streams all weights (%.0f MB) from HBM" % (nbytes / 1e6)},
            "roofline": {"bound": "tensor" if tensor_bound else "hbm", "kernel": f"VAE decode call ({launches} kernels)",
                         "achieved": flops / t_call / 1e12 if tensor_bound else nbytes / t_call / 1e9,
                         "peak": tf if tensor_bound else hbm, "unit": "TFLOP/s" if tensor_bound else "GB/s",
                         "frac": (flops / t_call / 1e12 / tf) if tensor_bound else (nbytes / t_call / 1e9 / hbm),
                         "peak_kind": peak_kind, "algorithmic_flops_per_call": flops,
                         "algorithmic_bytes_per_call": nbytes, "hbm_frac": nbytes / t_call / 1e9 / hbm, "traffic": None},
            "e2e": {"value": ws * T * args.steps / e2e_s, "unit": "latents/s", "h2d_bytes_per_step": T * 64 * 2,
                    "d2h_bytes_per_step": n_out * 4, "api": "ming_cuda_vae_decode (pinned host buffers)"},
            "gpu_launches": launches * args.steps, "clocks": ck, "cpu_baseline": cpu}


def run_loop(args, ws, rank, local):
    """BASELINE configs[4] through the library's loop entry (ming_cuda_loop_*,
    sampleLatents over B concurrent requests): per step, for every row, the
    adaLN flow head on the row's hidden state (10 Euler steps, CFG), the
    latent's projection into the next LM input and one LM decode step, as one
    CUDA graph; stop flags read back one step behind. The stop head's bias is
    set so that no request stops early: each runs its whole budget, as the
    config's fixed-length decode asks. One replica per GPU."""
    import torch

    import ming_b200 as M
    from ming_b200 import synth
    c = CONFIGS[args.config]
    B, P = c["batch"], c["prefill"]
    n_total = args.warmup + args.steps + 2
    max_ctx = ((P + n_total + 4 + 255) // 256) * 256
    pages = B * ((P + n_total + 4 + 15) // 16) + 16
    t0 = time.time()
    Wl = synth.lm_weights(seed=c["seed"], bits=c["bits"], layers=24)
    Wl["stop_head.bias"] = synth.f32_to_bf16(np.array([0.0, -30.0], np.float32))
    Wd = {**synth.ada_weights(seed=1), **synth.latent_proj_weights(seed=1)}
    log(f"[bench] weights generated in {time.time() - t0:.1f}s")
    cfg = M.default_cfg(weight_bits=c["bits"], dit_mode=M.DIT_ADALN, dit_hidden=768, dit_blocks=6, dit_heads=12,
                        dit_ff=3072, dit_frames=4, dit_max_batch=B, agg_blocks=0, max_ctx=max_ctx, max_pages=pages,
                        max_batch=B, max_seqs=B, max_prefill=max(512, min(2048, P)))
    ctx = M.Context(cfg, device=local, weights={**Wl, **Wd})
    params = M.sample_params(max_steps=n_total, max_len=P + n_total, cfg=2.0, temperature=0.0)
    lp = M.Loop(ctx, B, params)
    prompts = [synth.normal_bf16(c["seed"], f"bench.loop.prompt.{b}", (P, 896)) for b in range(B)]
    ctx.sync()
    t0 = time.time()
    ids = [lp.submit(prompts[b], None, seed=1000 + b) for b in range(B)]
    ctx.sync()
    log(f"[bench] prefill of {B} x {P} tokens in {time.time() - t0:.2f}s (submitted through the loop, host prompts)")
    for _ in range(args.warmup):
        a, q = lp.step()
        assert a == B and q == 0
    ctx.sync()
    stream = torch.cuda.ExternalStream(ctx.stream, device=local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    dist_barrier(ws)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    profile_range(True)
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        a, q = lp.step()
    ev1.record(stream)
    ev1.synchronize()
    host_s = time.perf_counter() - t0
    profile_range(False)
    dist_barrier(ws)
    ck = clocks.stop()
    assert a == B, "a request finished inside the timed steps"
    ms_local = ev0.elapsed_time(ev1)
    value, ms = aggregate_throughput(ms_local, B, args.steps, ws)
    lens_start = [P + args.warmup] * B
    # algorithmic bytes per step: LM weights + every sequence's KV once, the
    # head's weights once per Euler step, the projection
    wl, _ = algorithmic_bytes_lm(Wl, lens_start, B)
    kv = sum(12288 * (L + args.steps / 2.0 + 1) for L in lens_start)
    step_bytes = wl + kv + 10 * synth.nbytes(synth.ada_weights(seed=1)) + synth.nbytes(synth.latent_proj_weights(seed=1))
    hbm, tf, peak_kind = load_peaks()
    achieved = step_bytes / (ms_local / args.steps / 1e3) / 1e9
    # e2e: the host calls themselves (ming_cuda_loop_step: launch, the previous
    # step's flags read back), wall clock over the same K steps
    e2e_s = dist_max(host_s, ws)
    # launches per step: prep + flow head (run_dit's formula) + mean + projection + decode step + update
    R, NC = 8 * B, 2 * B
    lin = lambda rows, small=64: 1 if rows <= small else 2
    dit_launches = (lin(NC) + 10 + 7 * lin(10 * NC) + 10 * (lin(R, 8) + 6 * (4 * lin(R) + 1) + lin(R) + 1))
    launches = 1 + dit_launches + 2 + ctx.step_kernels(B) + 1
    lp.close()
    ctx.close()
    return {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 act / u4-g64 LM weights, bf16 head, f32 acc",
            "data": "synthetic (seeded random-init weights and N(0,1) embeddings, SplitMix64/Box-Muller; "
                    "stop head biased so no request stops early)",
            "config": {"workload": c["name"], "batch_per_gpu": B, "prompt_len": P,
                       "kv_positions_timed": [P + args.warmup, P + args.warmup + args.steps],
                       "token": "one request's loop step: its 10-step flow-head sample, projection and LM decode step",
                       "api": "ming_cuda_loop_submit / ming_cuda_loop_step (one CUDA graph per step)",
                       "parallelism": f"replicas x{ws} (no collective)",
                       "l2": "inputs larger than L2: every step streams all weights and the KV cache from HBM"},
            "roofline": {"bound": "hbm", "kernel": "loop step graph (flow head + projection + LM decode)",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_step": step_bytes, "traffic": None},
            "e2e": {"value": ws * B * args.steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 2 * B * 4 + 4,
                    "api": "ming_cuda_loop_step host calls, wall clock (inputs resident since submission; "
                           "per step the rows' stop flags and counts come back)"},
            "gpu_launches": launches * args.steps, "clocks": ck, "cpu_baseline": None}


def run_reference(args, ws, rank, local):
    """The reference's CPU path restated (oracle port, all host threads)."""
    if rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from ming_b200 import synth
    # every host thread this process may run on (torchrun sets OMP_NUM_THREADS=1)
    O.set_threads(len(os.sched_getaffinity(0)))
    cfgid = args.config
    c = CONFIGS[cfgid]
    if c.get("vae"):
        return run_reference_vae(args, ws, c, O)
    if c.get("dit") or c.get("loop"):
        return {"impl": "reference", "unavailable": "reference arm implemented for the LM-only configs"}
    B = c["batch"]
    lens = [c["prefill"]] * B if c["prefill"] else np.random.default_rng(c["seed"]).integers(32, 513, size=B).tolist()
    W = synth.lm_weights(seed=c["seed"], bits=c["bits"], layers=24)
    lm = O.Lm(W)
    nb = min(B, 2)
    caches, xs = [], []
    for b in range(nb):
        x = synth.normal_bf16(c["seed"], f"bench.prompt.{b}", (lens[b], 896))
        cch = lm.new_cache(lens[b] + args.warmup + args.steps + 8)
        out, _ = lm.forward(cch, x)
        caches.append(cch)
        xs.append(out[-1:])

    def step():
        for b in range(nb):
            xs[b], _ = lm.forward(caches[b], xs[b])

    for _ in range(args.warmup):
        step()
    budget = float(os.environ.get("MING_REF_BUDGET_S", "150"))
    n = 0
    t0 = time.perf_counter()
    while n < args.steps and (time.perf_counter() - t0) < budget:
        step()
        n += 1
    dt = time.perf_counter() - t0
    v = n * nb / dt
    return {"metric": METRIC, "value": v, "unit": "tokens/s", "impl": "reference", "n_gpus": ws, "steps": n,
            "warmup": args.warmup, "ms_per_step": dt / n * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 act / f32 acc (CPU)", "data": "synthetic",
            "config": {"workload": c["name"], "batch_per_gpu": B, "sequences_sampled": nb},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": O.threads(), "kind": "port",
                             "sample": f"{n} decode steps x {nb} sequence(s) of the workload (time-bounded at {budget:.0f}s)"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference_vae(args, ws, c, O):
    """The VAE decoder's CPU path restated (the oracle's f32 numpy decode, BLAS
    on all host threads): one decode of the fragment per step, time-bounded."""
    T = c["latents"]
    W, lat = vae_workload(c)
    for _ in range(min(args.warmup, 1)):
        O.vae_decode(W, lat, 24, window=64)
    budget = float(os.environ.get("MING_REF_BUDGET_S", "150"))
    n, t0 = 0, time.perf_counter()
    while n < args.steps and (n < 1 or time.perf_counter() - t0 < budget):
        O.vae_decode(W, lat, 24, window=64)
        n += 1
    dt = time.perf_counter() - t0
    v = n * T / dt
    return {"metric": "VAE decode latents/s (one 128-latent fragment per call)", "value": v, "unit": "latents/s",
            "impl": "reference", "n_gpus": ws, "steps": n, "warmup": args.warmup, "ms_per_step": dt / n * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (CPU)",
            "data": "synthetic", "config": {"workload": c["name"], "latents_per_call": T},
            "cpu_baseline": {"value": v, "unit": "latents/s", "cores": blas_threads(), "kind": "port",
                             "sample": f"{n} decode(s) of the workload's {T} latents (time-bounded at {budget:.0f}s)"},
            "e2e": {"value": v, "unit": "latents/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch32", action="store_true", help="config 2 only: skip the batch-32 (config 3) sub-measurement")
    ap.add_argument("--batch", type=int, default=None, help="override the config's batch (smaller profiling cases)")
    ap.add_argument("--prefill", type=int, default=None, help="override the config's prompt length")
    ap.add_argument("--e2e-api", choices=["decode", "noalloc"], default="decode",
                    help="entry point of the e2e loop (LM configs): ming_cuda_lm_decode or its allocation-free twin")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    c = CONFIGS[args.config]
    if args.batch is not None:
        c["batch"] = args.batch
        c["name"] += f" [batch overridden: {args.batch}]"
    if args.prefill is not None and c.get("prefill"):
        c["prefill"] = args.prefill
        c["name"] += f" [prefill overridden: {args.prefill}]"
    ws, rank, local = dist_setup(args) if args.impl == "ours" else (int(os.environ.get("WORLD_SIZE", "1")),
                                                                   int(os.environ.get("RANK", "0")),
                                                                   int(os.environ.get("LOCAL_RANK", "0")))
    if args.impl == "reference":
        res = run_reference(args, ws, rank, local)
    else:
        res = run_ours(args, ws, rank, local)
    if rank == 0 and res is not None:
        print(json.dumps(res), flush=True)
    if args.impl == "ours" and ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
