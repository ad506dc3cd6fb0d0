"""Per-step parity record of the LM token loop on BASELINE's own configs,
teacher-forced and free-running, GPU (through the C ABI) against the CPU
oracle. Needs a CUDA GPU; test infrastructure, not product code.

    python tests/parity_report.py --config 2 [--steps 1024] [--json out.json]

Configs (bench.py's workloads, same seeds, weights and prompts):
  1: bf16 LM, seed 0, N(0, 0.02) weights, 64-token prefill + 256 steps
  2: 4-bit g64 LM, seed 0, scales U(0.005, 0.02), 128-token prefill + 1024 steps

Teacher-forced (the reference's parity method, src/ming_parity.zig:6-8): every
step both sides take the oracle's previous output as input; recorded per
step: max-abs and cosine of the GPU output against the oracle's FUSED mode
(the reference's fused kernels), and each of GPU / FUSED / GRAPH (the
reference's plain MLX graph) against the oracle's F32 mode (no bf16 rounding).

Free-running (the reference parity tool's replay mode,
src/ming_parity.zig:204-235): each side feeds its own output back for the
whole loop; recorded per step: max-abs and cosine GPU vs oracle FUSED.
"""
import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "ming-tts-serve_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import ming_b200 as M  # noqa: E402
import oracle as O  # noqa: E402
from ming_b200 import synth  # noqa: E402

CONFIGS = {1: dict(bits=16, prefill=64, steps=256), 2: dict(bits=4, prefill=128, steps=1024)}


def f64(a):
    return synth.bf16_to_f32(a).astype(np.float64) if a.dtype == np.uint16 else np.asarray(a, np.float64)


def stats(a, b):
    a, b = f64(a).reshape(-1), f64(b).reshape(-1)
    return float(np.abs(a - b).max()), float((a * b).sum() / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


def rms(a, b):
    return float(np.sqrt(((f64(a).reshape(-1) - f64(b).reshape(-1)) ** 2).mean()))


def setup(cfgid, steps):
    c = CONFIGS[cfgid]
    W = synth.lm_weights(seed=0, bits=c["bits"], layers=24)
    n = c["prefill"] + steps + 2
    max_ctx = (n + 255) // 256 * 256
    cfg = M.default_cfg(weight_bits=c["bits"], dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=max_ctx,
                        max_pages=2 * (max_ctx // 16) + 8, max_batch=1, max_seqs=2, max_prefill=512)
    ctx = M.Context(cfg, weights=W)
    x = synth.normal_bf16(0, "bench.prompt.0", (c["prefill"], 896))
    return W, ctx, O.Lm(W), x, n


def teacher_forced(ctx, lm, x, steps, n, every=1):
    s = ctx.seq_alloc()
    cf, cg, ce = lm.new_cache(n), lm.new_cache(n), lm.new_cache(n)
    go, gst = ctx.prefill(s, x)
    fo, fst = lm.forward(cf, x)
    go_, _ = lm.forward(cg, x, O.MODE_GRAPH)
    eo = lm.forward_f32(ce, x)
    rows = []

    def rec(step, pos, g, f, gr, e, gs, fs):
        d, cs = stats(g[-1:], f[-1:])
        rows.append(dict(step=step, pos=pos, gpu_fused_maxabs=d, gpu_fused_cos=cs,
                         gpu_f32_maxabs=stats(g[-1:], e[-1:])[0], fused_f32_maxabs=stats(f[-1:], e[-1:])[0],
                         graph_f32_maxabs=stats(gr[-1:], e[-1:])[0], gpu_f32_cos=stats(g[-1:], e[-1:])[1],
                         fused_f32_cos=stats(f[-1:], e[-1:])[1], graph_f32_cos=stats(gr[-1:], e[-1:])[1],
                         gpu_f32_rms=rms(g[-1:], e[-1:]), fused_f32_rms=rms(f[-1:], e[-1:]),
                         graph_f32_rms=rms(gr[-1:], e[-1:]), stop_diff=float(abs(gs[-1] - fs[-1]))))

    rec(-1, x.shape[0] - 1, go, fo, go_, eo, gst, fst)
    xin = fo[-1:]
    for t in range(steps):
        pos = ctx.seq_len(s)
        g, gs = ctx.decode([s], xin)
        f, fs = lm.forward(cf, xin)
        gr, _ = lm.forward(cg, xin, O.MODE_GRAPH)
        e = lm.forward_f32(ce, xin)
        if t % every == 0 or t == steps - 1:
            rec(t, pos, g, f, gr, e, gs, fs)
        xin = f
    ctx.seq_free(s)
    return rows


def free_running(ctx, lm, x, steps, n):
    """GPU and oracle FUSED each feeding back their own outputs; beside them
    the oracle's GRAPH mode (the reference's plain MLX graph) free-running
    too: how far the reference's own two implementations drift apart."""
    s = ctx.seq_alloc()
    cf, cg = lm.new_cache(n), lm.new_cache(n)
    go, _ = ctx.prefill(s, x)
    fo, _ = lm.forward(cf, x)
    ro, _ = lm.forward(cg, x, O.MODE_GRAPH)
    gen, _ = ctx.generate([s], go[-1:], steps)
    rows = []
    xin, xg = fo[-1:], ro[-1:]
    for t in range(steps):
        f, _ = lm.forward(cf, xin)
        r, _ = lm.forward(cg, xg, O.MODE_GRAPH)
        d, cs = stats(gen[t], f)
        dg, cg_ = stats(r, f)
        rows.append(dict(step=t, pos=x.shape[0] + t, maxabs=d, cos=cs, graph_maxabs=dg, graph_cos=cg_))
        xin, xg = f, r
    ctx.seq_free(s)
    return rows


def summarize(tf, fr):
    a = lambda k: np.array([r[k] for r in tf])  # noqa: E731
    out = {"teacher_forced": {
        "steps": len(tf),
        "gpu_fused_maxabs_max": float(a("gpu_fused_maxabs").max()),
        "gpu_fused_maxabs_p50": float(np.median(a("gpu_fused_maxabs"))),
        "gpu_fused_cos_min": float(a("gpu_fused_cos").min()),
        "steps_over_2e-2": int((a("gpu_fused_maxabs") > 2e-2).sum()),
        "steps_cos_below_0.999": int((a("gpu_fused_cos") <= 0.999).sum()),
        "gpu_f32_maxabs_max": float(a("gpu_f32_maxabs").max()),
        "fused_f32_maxabs_max": float(a("fused_f32_maxabs").max()),
        "graph_f32_maxabs_max": float(a("graph_f32_maxabs").max()),
        "steps_gpu_further_from_f32_than_fused": int((a("gpu_f32_maxabs") > a("fused_f32_maxabs")).sum()),
        "steps_gpu_further_from_f32_than_both": int(
            (a("gpu_f32_maxabs") > np.maximum(a("fused_f32_maxabs"), a("graph_f32_maxabs"))).sum()),
        "stop_diff_max": float(a("stop_diff").max()),
        "gpu_f32_rms_over_ref_max": float((a("gpu_f32_rms") / np.maximum(a("fused_f32_rms"), a("graph_f32_rms"))).max()),
        "gpu_f32_maxabs_over_ref_max": float((a("gpu_f32_maxabs") /
                                              np.maximum(a("fused_f32_maxabs"), a("graph_f32_maxabs"))).max()),
        "gpu_f32_cos_deficit_max": float((np.minimum(a("fused_f32_cos"), a("graph_f32_cos")) - a("gpu_f32_cos")).max()),
        "worst": sorted(tf, key=lambda r: -r["gpu_fused_maxabs"])[:5],
    }}
    if fr:
        m = np.array([r["maxabs"] for r in fr])
        c = np.array([r["cos"] for r in fr])
        gm = np.array([r["graph_maxabs"] for r in fr])
        gc = np.array([r["graph_cos"] for r in fr])
        marks = sorted({0, 1, 3, 7, 15, 31, 63, 127, 255, 511, len(fr) - 1} & set(range(len(fr))))
        first = lambda v: int(np.argmax(v <= 0.999)) if (v <= 0.999).any() else None  # noqa: E731
        out["free_running"] = {"steps": len(fr),
                               "at": {str(i): {"gpu_vs_fused": [float(m[i]), float(c[i])],
                                               "graph_vs_fused": [float(gm[i]), float(gc[i])]} for i in marks},
                               "gpu_first_cos_below_0.999": first(c), "graph_first_cos_below_0.999": first(gc)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--no-free", action="store_true")
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    steps = a.steps or CONFIGS[a.config]["steps"]
    O.set_threads(len(os.sched_getaffinity(0)))
    t0 = time.time()
    W, ctx, lm, x, n = setup(a.config, steps)
    tf = teacher_forced(ctx, lm, x, steps, n)
    fr = None if a.no_free else free_running(ctx, lm, x, steps, n)
    ctx.close()
    res = {"config": a.config, "steps": steps, "oracle_threads": O.threads(), "wall_s": time.time() - t0, **summarize(tf, fr)}
    print(json.dumps(res, indent=1))
    if a.json:
        with open(a.json, "w") as f:
            json.dump({"summary": res, "teacher_forced_rows": tf, "free_running_rows": fr}, f)


if __name__ == "__main__":
    main()
