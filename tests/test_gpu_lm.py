"""GPU parity of the LM decode path through the C ABI against the CPU oracle.

Tolerance (the benchmark's stated bf16 tolerance): per-step post-norm hidden states within
max-abs 2e-2 and cosine > 0.999 (bf16), gated on teacher-forced steps (both
sides get the oracle's input each step, as the reference's parity tool does,
src/ming_parity.zig:6-8). Integer work — KV placement through the block table
and quantized-weight unpacking — is compared bit for bit.

Conditioning: with the benchmark's 4-bit init (uniform codes, scales
U(0.005, 0.02): weight std ~0.058) attention scores are large and peaky, and a
bf16 rounding difference can move a row's attention to another position: the
oracle's own fused and plain-graph rounding modes then disagree on a few rows
by O(1). The strict gates therefore run 4/8-bit models with scales
U(0.002, 0.005) (weight std ~0.016, like the bf16 config); the benchmark's
distribution is gated against that fused-vs-graph spread instead
(test_q4_baseline_init_within_reference_spread).
"""
QS = (0.002, 0.005)  # well-conditioned 4/8-bit group scales for the strict gates
import numpy as np
import pytest

import ming_b200 as M
import oracle as O
from ming_b200 import synth

from conftest import as_accurate_as_reference, bf, bf16_ulp, close, within_reference

pytestmark = pytest.mark.gpu

TOL, COS = 2e-2, 0.999


def make_ctx(W, bits, layers, **kw):
    cfg = M.default_cfg(layers=layers, weight_bits=bits, dit_mode=M.DIT_NONE, agg_blocks=0, **kw)
    return M.Context(cfg, weights=W)


@pytest.fixture(scope="module")
def q4_24(cuda_ok):
    W = synth.lm_weights(seed=0, bits=4, layers=24, qscale=QS)
    ctx = make_ctx(W, 4, 24, max_ctx=2048, max_pages=1024, max_batch=32)
    yield W, ctx, O.Lm(W)
    ctx.close()


@pytest.mark.parametrize("bits", [4, 8, 16])
def test_unpack_bit_exact(cuda_ok, bits):
    W = synth.lm_weights(seed=1, bits=bits, layers=1)
    ctx = make_ctx(W, bits, 1)
    for n, (o, i) in {"self_attn.q_proj": (896, 896), "self_attn.k_proj": (128, 896), "self_attn.v_proj": (128, 896),
                      "self_attn.o_proj": (896, 896), "mlp.gate_proj": (4864, 896), "mlp.up_proj": (4864, 896),
                      "mlp.down_proj": (896, 4864)}.items():
        p = f"model.model.layers.0.{n}"
        got = ctx.unpack_linear(p + ".weight", o, i)
        ref = O.lin_dequant(W, p)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), n
    ctx.close()


def _teacher_forced(ctx, lm, x_prompt, steps, seed):
    """Prefill both, then `steps` decode steps, each fed the oracle's previous
    output. The oracle runs twice: fused rounding (the reference's fused
    kernels, the parity target) and plain-graph rounding (the reference's MLX
    graph), which sets the spread `within_reference` allows. Returns per-step
    (maxabs, cos, ok) lists."""
    s = ctx.seq_alloc()
    n = x_prompt.shape[0] + steps + 1
    cache, cache_g = lm.new_cache(n), lm.new_cache(n)
    go, gs = ctx.prefill(s, x_prompt)
    ro, rs = lm.forward(cache, x_prompt)
    rg, _ = lm.forward(cache_g, x_prompt, O.MODE_GRAPH)
    res = [within_reference(go, ro, rg)]
    assert np.abs(gs - rs).max() < 1e-2
    x = ro[-1:]
    for t in range(steps):
        go, gs = ctx.decode([s], x)
        ro, rs = lm.forward(cache, x)
        rg, _ = lm.forward(cache_g, x, O.MODE_GRAPH)
        res.append(within_reference(go, ro, rg))
        assert abs(gs[0] - rs[0]) < 1e-2
        x = ro
    ctx.seq_free(s)
    return res


def test_decode_parity_q4_full_model(q4_24):
    W, ctx, lm = q4_24
    x = synth.normal_bf16(0, "test.prompt.q4", (64, 896))
    res = _teacher_forced(ctx, lm, x, 8, 0)
    for i, (d, c, ok) in enumerate(res):
        assert ok, f"step {i}: maxabs {d:.4g} cos {c:.6f}"


@pytest.mark.parametrize("bits,layers", [(16, 6), (8, 6)])
def test_decode_parity_bf16_q8(cuda_ok, bits, layers):
    W = synth.lm_weights(seed=2, bits=bits, layers=layers, qscale=QS)
    ctx = make_ctx(W, bits, layers)
    x = synth.normal_bf16(1, "test.prompt", (37, 896))
    res = _teacher_forced(ctx, O.Lm(W), x, 6, 1)
    for i, (d, c, ok) in enumerate(res):
        assert ok, f"step {i}: maxabs {d:.4g} cos {c:.6f}"
    ctx.close()


def test_prefill_bf16_many_rows(cuda_ok):
    """bf16 weights with 96 prompt rows: the projections run on the tcgen05
    linear (64+ rows), gated like the other multi-layer outputs."""
    W = synth.lm_weights(seed=3, bits=16, layers=2)
    ctx = make_ctx(W, 16, 2)
    res = _teacher_forced(ctx, O.Lm(W), synth.normal_bf16(3, "test.prompt.bf16.96", (96, 896)), 2, 3)
    for i, (d, c, ok) in enumerate(res):
        assert ok, f"step {i}: maxabs {d:.4g} cos {c:.6f}"
    ctx.close()


@pytest.mark.parametrize("bits", [4, 8])
def test_prefill_quantized_tcgen05_many_rows(cuda_ok, bits):
    """4/8-bit weights with 200 prompt rows: chunks above 64 rows run on the
    tcgen05 linear over the weights' f16 hi | lo prefill copies (the rows
    staged in f16 as the mma.sync kernels stage them), gated like the other
    multi-layer outputs."""
    W = synth.lm_weights(seed=4, bits=bits, layers=2, qscale=QS)
    ctx = make_ctx(W, bits, 2)
    res = _teacher_forced(ctx, O.Lm(W), synth.normal_bf16(4, f"test.prompt.q{bits}.200", (200, 896)), 2, 3)
    for i, (d, c, ok) in enumerate(res):
        assert ok, f"step {i}: maxabs {d:.4g} cos {c:.6f}"
    ctx.close()


def test_batched_decode_ragged_prompts(q4_24):
    W, ctx, lm = q4_24
    lens = [1, 17, 40, 64, 300]
    seqs, caches, xs = [], [], []
    for i, L in enumerate(lens):
        s = ctx.seq_alloc()
        x = synth.normal_bf16(3, f"test.ragged.{i}", (L, 896))
        c = lm.new_cache(L + 8)
        ctx.prefill(s, x, want_out=False)
        ro, _ = lm.forward(c, x)
        seqs.append(s)
        caches.append(c)
        xs.append(ro[-1])
    x = np.stack(xs)
    for t in range(3):
        go, gs = ctx.decode(seqs, x)
        ref = []
        for b in range(len(lens)):
            ro, rs = lm.forward(caches[b], x[b:b + 1])
            ref.append(ro[0])
            assert abs(gs[b] - rs[0]) < 1e-2
        ref = np.stack(ref)
        d, c, ok = close(go, ref)
        assert ok, f"step {t}: maxabs {d:.4g} cos {c:.6f}"
        x = ref
    for s in seqs:
        ctx.seq_free(s)


@pytest.mark.parametrize("bits,B,gains", [(4, 20, False), (4, 40, False), (8, 12, False), (16, 33, False), (4, 24, True)])
def test_batched_decode_many_rows(cuda_ok, bits, B, gains):
    """Decode batches of 9..64 rows run on the decode-batch linear (bulk
    weight copies, K split over thread-block clusters, 32-row blocks): B = 40
    and 33 take two row blocks. Prompts of 1..30 rows also put the prefill
    chunks above 8 rows on it. Teacher-forced against the oracle per row,
    gated like the other multi-layer outputs (the oracle's fused rounding,
    widened by its fused-vs-graph spread, or no further from the oracle's
    f32 mode than the reference paths are); replaying the same step gives the
    same bits (the cluster reduction sums in a fixed order). `gains`: RMSNorm
    gains drawn from U(0.5, 1.5) instead of 1 (the staged rows are scaled)."""
    layers = 3
    W = synth.lm_weights(seed=11, bits=bits, layers=layers, qscale=QS)
    if gains:
        g = np.random.default_rng(5)
        for l in range(layers):
            for n in ("input_layernorm", "post_attention_layernorm"):
                v = g.uniform(0.5, 1.5, 896).astype(np.float32)
                W[f"model.model.layers.{l}.{n}.weight"] = (v.view(np.uint32) >> 16).astype(np.uint16)
    ctx = make_ctx(W, bits, layers, max_ctx=256, max_pages=1024, max_batch=64, max_seqs=64)
    lm = O.Lm(W)
    rng = np.random.default_rng(B)
    lens = rng.integers(1, 31, size=B).tolist()
    seqs, caches, gcaches, fcaches, xs = [], [], [], [], []
    for i, L in enumerate(lens):
        s = ctx.seq_alloc()
        x = synth.normal_bf16(7, f"test.many.{bits}.{B}.{gains}.{i}", (L, 896))
        c, cg, cf = lm.new_cache(L + 4), lm.new_cache(L + 4), lm.new_cache(L + 4)
        got, _ = ctx.prefill(s, x)
        ro, _ = lm.forward(c, x)
        rg, _ = lm.forward(cg, x, O.MODE_GRAPH)
        rf = lm.forward_f32(cf, x)
        d, cs, ok = within_reference(got, ro, rg, exact=rf)
        assert ok, f"prefill row {i} (L={L}): maxabs {d:.4g} cos {cs:.6f}"
        seqs.append(s)
        caches.append(c)
        gcaches.append(cg)
        fcaches.append(cf)
        xs.append(ro[-1])
    x = np.stack(xs)
    for t in range(2):
        go, gs = ctx.decode(seqs, x)
        ref, refg, reff, rstop = [], [], [], []
        for b in range(B):
            ro, rs = lm.forward(caches[b], x[b:b + 1])
            rg, _ = lm.forward(gcaches[b], x[b:b + 1], O.MODE_GRAPH)
            reff.append(lm.forward_f32(fcaches[b], x[b:b + 1])[0])
            ref.append(ro[0])
            refg.append(rg[0])
            rstop.append(rs[0])
        ref = np.stack(ref)
        d, cs, ok = within_reference(go, ref, np.stack(refg), exact=np.stack(reff))
        assert ok, f"step {t}: maxabs {d:.4g} cos {cs:.6f}"
        assert np.abs(gs - np.array(rstop)).max() < 1e-2
        if t == 0:  # the same step again, from the same cache state
            for q, L in zip(seqs, lens):
                ctx.seq_truncate(q, L)
            go2, gs2 = ctx.decode(seqs, x)
            assert np.array_equal(go, go2) and np.array_equal(gs, gs2)
        x = ref
    ctx.close()


@pytest.mark.parametrize("bits,B,gains", [(4, 20, False), (8, 12, False), (4, 40, False), (4, 12, True)])
def test_batched_decode_tcgen05(cuda_ok, monkeypatch, bits, B, gains):
    """The decode-batch linear's tcgen05 variant forced on every projection
    (MING_BULK_TC=1: codes dequantized into 128-byte-swizzled weight blocks,
    one tensor-memory accumulator per K group, the group scale and bias in
    f32; `gains`: non-unit RMSNorm gains, two operand parts), gated like the
    mma.sync variant against the oracle."""
    monkeypatch.setenv("MING_BULK_TC", "1")
    layers = 2
    W = synth.lm_weights(seed=12, bits=bits, layers=layers, qscale=QS)
    if gains:
        g = np.random.default_rng(6)
        for l in range(layers):
            for n in ("input_layernorm", "post_attention_layernorm"):
                v = g.uniform(0.5, 1.5, 896).astype(np.float32)
                W[f"model.model.layers.{l}.{n}.weight"] = (v.view(np.uint32) >> 16).astype(np.uint16)
    ctx = make_ctx(W, bits, layers, max_ctx=256, max_pages=1024, max_batch=64, max_seqs=64)
    lm = O.Lm(W)
    lens = np.random.default_rng(B + 1).integers(1, 24, size=B).tolist()
    seqs, caches, gcaches, fcaches, xs = [], [], [], [], []
    for i, L in enumerate(lens):
        s = ctx.seq_alloc()
        x = synth.normal_bf16(8, f"test.tc.{bits}.{B}.{gains}.{i}", (L, 896))
        c, cg, cf = lm.new_cache(L + 2), lm.new_cache(L + 2), lm.new_cache(L + 2)
        got, _ = ctx.prefill(s, x)
        ro, _ = lm.forward(c, x)
        rg, _ = lm.forward(cg, x, O.MODE_GRAPH)
        rf = lm.forward_f32(cf, x)
        d, cs, ok = within_reference(got, ro, rg, exact=rf)
        assert ok, f"prefill row {i} (L={L}): maxabs {d:.4g} cos {cs:.6f}"
        seqs.append(s)
        caches.append(c)
        gcaches.append(cg)
        fcaches.append(cf)
        xs.append(ro[-1])
    x = np.stack(xs)
    go, gs = ctx.decode(seqs, x)
    ref, refg, reff = [], [], []
    for b in range(B):
        ref.append(lm.forward(caches[b], x[b:b + 1])[0][0])
        refg.append(lm.forward(gcaches[b], x[b:b + 1], O.MODE_GRAPH)[0][0])
        reff.append(lm.forward_f32(fcaches[b], x[b:b + 1])[0])
    d, cs, ok = within_reference(go, np.stack(ref), np.stack(refg), exact=np.stack(reff))
    assert ok, f"decode: maxabs {d:.4g} cos {cs:.6f}"
    ctx.close()


def test_generate_matches_decode_loop_bitwise(q4_24):
    W, ctx, lm = q4_24
    x = synth.normal_bf16(4, "test.gen", (20, 896))
    a, b = ctx.seq_alloc(), ctx.seq_alloc()
    oa, _ = ctx.prefill(a, x)
    ob, _ = ctx.prefill(b, x)
    assert np.array_equal(oa, ob)
    gen, gstop = ctx.generate([a], oa[-1:], 6)
    xin = ob[-1:]
    for t in range(6):
        o, st = ctx.decode([b], xin)
        assert np.array_equal(o, gen[t]), t
        assert np.array_equal(st, gstop[t]), t
        xin = o
    # determinism: regenerate from the same prefix
    ctx.seq_truncate(a, 20)
    gen2, _ = ctx.generate([a], oa[-1:], 6)
    assert np.array_equal(gen, gen2)
    ctx.seq_free(a)
    ctx.seq_free(b)


def test_long_context_split_and_page_boundaries(cuda_ok):
    W = synth.lm_weights(seed=7, bits=4, layers=2, qscale=QS)
    ctx = make_ctx(W, 4, 2, max_prefill=96)  # prefill runs in chunks of 96 rows
    lm = O.Lm(W)
    x = synth.normal_bf16(8, "test.long", (510, 896))
    s = ctx.seq_alloc()
    c, cg = lm.new_cache(530), lm.new_cache(530)
    go, _ = ctx.prefill(s, x)
    ro, _ = lm.forward(c, x)
    rg, _ = lm.forward(cg, x, O.MODE_GRAPH)
    d, cs, ok = within_reference(go, ro, rg)
    assert ok, (d, cs)
    xin = ro[-1:]
    for t in range(6):  # positions 510..515 cross the 512 split boundary
        go, _ = ctx.decode([s], xin)
        ro, _ = lm.forward(c, xin)
        rg, _ = lm.forward(cg, xin, O.MODE_GRAPH)
        d, cs, ok = within_reference(go, ro, rg)
        assert ok, (t, d, cs)
        xin = ro
    ctx.close()


def test_errors_are_reported(q4_24):
    W, ctx, lm = q4_24
    with pytest.raises(M.MingError):
        ctx.decode([999], np.zeros((1, 896), np.uint16))
    s = ctx.seq_alloc()
    with pytest.raises(M.MingError):  # decode before any prefill
        ctx.decode([s], np.zeros((1, 896), np.uint16))
    ctx.prefill(s, np.zeros((2, 896), np.uint16), want_out=False)
    with pytest.raises(M.MingError):  # same sequence twice in a batch
        ctx.decode([s, s], np.zeros((2, 896), np.uint16))
    ctx.seq_free(s)


def test_q4_baseline_init_prefill(cuda_ok):
    """The benchmark's 4-bit distribution (scales U(0.005, 0.02)) on a 100-row
    prefill of 2 layers (the tcgen05 linear over the f16 hi | lo prefill
    copies). Its peaky attention makes the reference's own FUSED and GRAPH
    paths differ by 0.02-0.63 max-abs on some rows (one row's attention
    flips), so the strict 2e-2 cannot hold against either: every row is
    gated by within_reference (the tolerance or twice that row's reference
    spread, cosine > 0.999 or the reference's own) and is as accurate as the
    reference against exact arithmetic (oracle F32 mode). Measured on the
    flipping row (cosine to exact): tcgen05 0.8893, mma.sync 0.8856, FUSED
    0.8891."""
    W = synth.lm_weights(seed=7, bits=4, layers=2)
    ctx = make_ctx(W, 4, 2)
    lm = O.Lm(W)
    x = synth.normal_bf16(8, "dbg.100", (100, 896))
    s = ctx.seq_alloc()
    go, _ = ctx.prefill(s, x)
    fused = lm.forward(lm.new_cache(104), x, O.MODE_FUSED)[0]
    graph = lm.forward(lm.new_cache(104), x, O.MODE_GRAPH)[0]
    exact = lm.forward_f32(lm.new_cache(104), x)
    d, c, ok = within_reference(go, fused, graph, exact=exact)
    assert ok, (d, c)
    rr, mr, cd, ok = as_accurate_as_reference(go, fused, graph, exact)
    assert ok, (rr, mr, cd)
    ctx.close()
