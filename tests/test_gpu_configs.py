"""Teacher-forced parity on BASELINE's own LM configs at full size, 24 layers,
through the C ABI against the oracle (the reference's parity method: both
sides take the oracle's previous output each step, src/ming_parity.zig:6-8).

Config 2 (the headline: 4-bit g64, scales U(0.005, 0.02), 128-token prompt,
1,024 decode steps to position 1,152): every decode step is gated at the
north star's bf16 tolerance: max-abs 2e-2 (two bf16 steps where |v| >= 2)
and cosine > 0.999 against the oracle's FUSED mode, p(stop) within 1e-2.
The 128 prompt rows (the prefill, on the tiled many-row linear) meet cosine
> 0.999 but reach 0.031 max-abs on some rows, where the reference's own
FUSED and GRAPH paths differ by as much: they are gated like the other
many-row outputs (within_reference), and as accurate as the reference
against exact arithmetic.

Config 1 (bf16, N(0, 0.02) weights, 64-token prompt, 256 steps): the
reference's own fused kernels are 0.094 max-abs away from exact f32
arithmetic on this model (oracle FUSED vs F32 mode), so no implementation
that rounds where the reference does can be held to 2e-2 against any one of
them. Gate: cosine > 0.999 against FUSED (the north star's cosine), and the
GPU no less accurate than the reference: per step its distance to the
oracle's F32 result within 1.5x the farther of the reference's two paths
(FUSED, GRAPH) in RMS, 2x in max-abs, and its cosine to F32 no lower than
theirs minus 1e-4.
"""
import numpy as np
import pytest

import ming_b200 as M
import oracle as O
from ming_b200 import synth

from conftest import as_accurate_as_reference, bf, close, within_reference

pytestmark = pytest.mark.gpu


def _setup(bits, prefill, steps):
    W = synth.lm_weights(seed=0, bits=bits, layers=24)
    n = prefill + steps + 2
    max_ctx = (n + 255) // 256 * 256
    cfg = M.default_cfg(weight_bits=bits, dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=max_ctx, max_pages=max_ctx // 16 + 8,
                        max_batch=1, max_seqs=1, max_prefill=512)
    ctx = M.Context(cfg, weights=W)
    return ctx, O.Lm(W), synth.normal_bf16(0, "bench.prompt.0", (prefill, 896)), n


def test_config2_q4_baseline_init_1024_steps(cuda_ok):
    ctx, lm, x, n = _setup(4, 128, 1024)
    s = ctx.seq_alloc()
    cache = lm.new_cache(n)
    go, gs = ctx.prefill(s, x)
    ro, rs = lm.forward(cache, x)
    rg, _ = lm.forward(lm.new_cache(n), x, O.MODE_GRAPH)
    re_ = lm.forward_f32(lm.new_cache(n), x)
    d, c, ok = within_reference(go, ro, rg, exact=re_)
    assert ok, ("prefill", d, c)
    rr, mr, cd, ok = as_accurate_as_reference(go, ro, rg, re_)
    assert ok, ("prefill accuracy", rr, mr, cd)
    assert np.abs(gs - rs).max() < 1e-2
    xin = ro[-1:]
    worst = (0.0, 1.0)
    for t in range(1024):
        g, gs = ctx.decode([s], xin)
        r, rs = lm.forward(cache, xin)
        d, c, ok = close(g, r)
        assert ok, f"step {t} (position {128 + t}): maxabs {d:.4g} cos {c:.6f}"
        assert abs(gs[0] - rs[0]) < 1e-2, t
        worst = (max(worst[0], d), min(worst[1], c))
        xin = r
    assert ctx.seq_len(s) == 128 + 1024
    ctx.close()
    print("config 2 worst step: maxabs %.4g cos %.7f" % worst)


def test_config1_bf16_24_layers_256_steps(cuda_ok):
    ctx, lm, x, n = _setup(16, 64, 256)
    s = ctx.seq_alloc()
    cf, cg, ce = lm.new_cache(n), lm.new_cache(n), lm.new_cache(n)
    go, _ = ctx.prefill(s, x)
    fo, _ = lm.forward(cf, x)
    lm.forward(cg, x, O.MODE_GRAPH)
    lm.forward_f32(ce, x)

    def cos(a, b):
        return float((a * b).sum() / (np.linalg.norm(a) * np.linalg.norm(b)))

    xin = fo[-1:]
    worst = {"cos_fused": 1.0, "rms_ratio": 0.0, "max_ratio": 0.0, "cos_deficit": -1.0, "maxabs_fused": 0.0}
    for t in range(256):
        g, gs = ctx.decode([s], xin)
        f, fs = lm.forward(cf, xin)
        r, _ = lm.forward(cg, xin, O.MODE_GRAPH)
        e = lm.forward_f32(ce, xin).astype(np.float64).reshape(-1)
        gv, fv, rv = bf(g).reshape(-1), bf(f).reshape(-1), bf(r).reshape(-1)
        c_gf = cos(gv, fv)
        rms = lambda a: float(np.sqrt(((a - e) ** 2).mean()))  # noqa: E731
        rms_ratio = rms(gv) / max(rms(fv), rms(rv))
        max_ratio = np.abs(gv - e).max() / max(np.abs(fv - e).max(), np.abs(rv - e).max())
        cos_def = min(cos(fv, e), cos(rv, e)) - cos(gv, e)
        msg = (f"step {t}: cos vs fused {c_gf:.6f}, rms/ref {rms_ratio:.3f}, max/ref {max_ratio:.3f}, "
               f"cos deficit {cos_def:.2e}, maxabs vs fused {np.abs(gv - fv).max():.4g}")
        assert c_gf > 0.999, msg
        assert rms_ratio <= 1.5 and max_ratio <= 2.0 and cos_def <= 1e-4, msg
        assert abs(gs[0] - fs[0]) < 1e-2, msg
        worst = {"cos_fused": min(worst["cos_fused"], c_gf), "rms_ratio": max(worst["rms_ratio"], rms_ratio),
                 "max_ratio": max(worst["max_ratio"], max_ratio), "cos_deficit": max(worst["cos_deficit"], cos_def),
                 "maxabs_fused": max(worst["maxabs_fused"], float(np.abs(gv - fv).max()))}
        xin = f
    ctx.close()
    print("config 1 worst step:", worst)
