"""Per-phase timeline of the persistent decode kernel (diagnostics).

Run on a GPU from the repository root:

    python ming-tts-serve_b200/ming_b200/mega_trace.py [--prompt 640] [--layers 24]

It builds a 4-bit batch-1 context with MING_MEGA_TRACE=1 (each CTA of the
persistent kernel then writes clock64 stamps per layer), prefills a seeded
prompt, runs 8 decode steps and prints, for the middle layers of the last
step, when each phase boundary is reached relative to the CTA's own layer
start (clock64 counts per SM), median and maximum over the CTAs, followed by
the GEMV sub-steps and the per-warp gate|up / down stamps. Stamp slots:
0 layer start, 1/2 q|k|v stage start/end, 9 attention items done, 3/4 o_proj,
5/6 gate|up, 7/8 down, 10 + 7q + k sub-step k of GEMV phase q, 40-55 the end
of each of the first 8 warps' runs in gate|up (40-47) and down (48-55), 56-63
their first gate|up slot in hand.
"""
import argparse
import ctypes
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

SLOTS = 64  # stamp slots per (CTA, layer), as the kernel writes them


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt", type=int, default=640)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--sm-ghz", type=float, default=1.965, help="SM clock used to turn cycles into microseconds")
    args = ap.parse_args()
    os.environ["MING_MEGA_TRACE"] = "1"  # read when the context is finalized
    import numpy as np

    import ming_b200 as M
    from ming_b200 import synth

    layers = args.layers
    W = synth.lm_weights(seed=0, bits=4, layers=layers)
    cfg = M.default_cfg(layers=layers, weight_bits=4, dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=2048, max_pages=1024)
    ctx = M.Context(cfg, device=0, weights=W)
    s = ctx.seq_alloc()
    ctx.prefill(s, synth.normal_bf16(0, "trace.prompt", (args.prompt, 896)))
    x = synth.normal_bf16(9, "trace.x", (1, 896))
    for _ in range(8):
        x, _ = ctx.decode([s], x)
    ctx.sync()
    L = M.lib()
    L.ming_cuda_debug_trace.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    n = ctypes.c_int(0)
    sms = 148
    buf = np.zeros((sms, layers, SLOTS), dtype=np.int64)
    rc = L.ming_cuda_debug_trace(ctx._h, buf.ctypes.data, buf.size, ctypes.byref(n))
    if rc != 0 or n.value <= 0:
        raise SystemExit(f"no persistent-kernel trace (rc {rc}, n {n.value}): {L.ming_cuda_last_error()}")
    t = buf[: n.value].astype(np.float64)
    us = 1.0 / (args.sm_ghz * 1e3)
    mid = range(2, layers - 2)
    names = {1: "q0 stage start (after await+resid)", 2: "q0 end", 9: "P1 attention items done",
             3: "q1 stage start (combine done)", 4: "q1 end", 5: "q2 stage start (after await+resid)", 6: "q2 end",
             7: "q3 stage start (after await h)", 8: "q3 end"}
    for k, nm in names.items():
        v = [(t[:, l, k] - t[:, l, 0]) * us for l in mid]
        print(f"{nm:40s} median {np.mean([np.median(x) for x in v]):6.2f} us  max {np.mean([x.max() for x in v]):6.2f} us")
    v = [(t[:, l + 1, 0] - t[:, l, 0]) * us for l in mid]
    print(f"{'next layer start':40s} median {np.mean([np.median(x) for x in v]):6.2f} us  max {np.mean([x.max() for x in v]):6.2f} us")
    for q in range(4):
        for kk in range(5):
            v = [np.median(t[:, l, 10 + 7 * q + kk] - t[:, l, 1 + 2 * q]) * us for l in mid]
            print(f"  phase {q} sub {kk}: median {np.mean(v):6.2f} us after stage start")
    for w in range(8):
        a = [np.median(t[:, l, 56 + w] - t[:, l, 5]) * us for l in mid]
        b = [np.median(t[:, l, 40 + w] - t[:, l, 5]) * us for l in mid]
        c = [np.median(t[:, l, 48 + w] - t[:, l, 7]) * us for l in mid]
        print(f"  warp {w}: gu first data {np.mean(a):6.2f}  gu run done {np.mean(b):6.2f}  "
              f"down run done {np.mean(c):6.2f} us after stage start")
    ctx.close()


if __name__ == "__main__":
    main()
