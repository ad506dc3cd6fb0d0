"""bench.py's work accounting on CPU: the VAE decoder's algorithmic FLOPs and
bytes per call (the numerators of its roofline line), checked against the
count written out by hand for a small decoder."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from ming_b200 import synth  # noqa: E402


def test_vae_work_counts_linears_attention_and_bytes():
    H, FF, L, T = 896, 128, 2, 20
    W = synth.vae_weights(seed=3, layers=L, ff=FF)
    flops, nbytes = bench.vae_work(W, T)
    F = 4 * T
    # q, k, v, o, gate, up, down of one layer (14 query heads, 2 kv heads of 64)
    layer = H * H + 2 * (128 * H) + H * H + 2 * (FF * H) + H * FF
    # scores and P.V: 2 FLOPs per dim and key each, 14 heads, row i sees min(i + 1, 64) keys
    att = 4 * 64 * 14 * sum(min(i + 1, 64) for i in range(F))
    want = 2 * T * (H * 64) + 2 * F * (L * layer + 3530 * H) + L * att
    assert flops == want
    assert nbytes == sum(v.nbytes for v in W.values()) + T * 64 * 2 + F * 882 * 4


def test_vae_config_is_the_bench_workload():
    c = bench.CONFIGS[6]
    assert c.get("vae") and c["latents"] == 128
    assert bench.blas_threads() >= 1
    assert np.isfinite(bench.vae_work(synth.vae_weights(seed=3, layers=1, ff=64), 2)[0])
