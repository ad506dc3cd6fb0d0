"""KV-cache placement and long-context attention, bit for bit where the work is
integer indexing.

The paged pool ([page][layer][K|V][kv_head][16][64] bf16, a block table per
sequence) replaces the reference's per-step cache concatenation
(src/ming_model.zig:595-604,638-662). ming_cuda_kv_write stores known values
through the same device index function the decode kernels append with, and
ming_cuda_kv_read reads them back with an independent host-side formula:

* a write/read round trip over interleaved pages is bit-exact;
* a decode step leaves every cached position of every sequence bit-identical
  and writes its new position into that sequence's own slot (compared with
  the oracle's appended K/V within the bf16 tolerance, since the GEMV's f32
  summation order differs);
* attention over an injected cache of up to 4,500 positions (the persistent
  kernel's 128-position chunks, and the per-kernel path's split kernel plus
  combine kernel above 8 splits of 256) matches the oracle reading the same
  cache values.
"""
import numpy as np
import pytest

import ming_b200 as M
import oracle as O
from ming_b200 import synth

from conftest import bf, bf16_ulp, close

pytestmark = pytest.mark.gpu

QS = (0.002, 0.005)


def _model(layers, max_ctx, max_batch=8):
    W = synth.lm_weights(seed=21, bits=4, layers=layers, qscale=QS)
    cfg = M.default_cfg(layers=layers, weight_bits=4, dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=max_ctx,
                        max_pages=4096, max_batch=max_batch, max_seqs=16)
    return W, M.Context(cfg, weights=W), O.Lm(W)


def _inject(ctx, lm_caches, seqs, lens, layers, tag, chunk=96):
    """Writes random caches for every (sequence, layer), chunk by chunk with
    the sequences interleaved so their physical pages interleave; mirrors the
    values into the oracle caches. Returns {seq: (K, V)} [layers][2][n][64]."""
    vals = {}
    for s, n in zip(seqs, lens):
        K = np.stack([synth.normal_bf16(3, f"{tag}.{s}.{l}.k", (2, n, 64)) for l in range(layers)])
        V = np.stack([synth.normal_bf16(3, f"{tag}.{s}.{l}.v", (2, n, 64)) for l in range(layers)])
        vals[s] = (K, V)
    done = {s: 0 for s in seqs}
    while any(done[s] < n for s, n in zip(seqs, lens)):
        for s, n in zip(seqs, lens):
            p0 = done[s]
            if p0 >= n:
                continue
            p1 = min(n, p0 + chunk)
            K, V = vals[s]
            for l in range(layers):
                ctx.kv_write(s, l, p0, K[l, :, p0:p1], V[l, :, p0:p1])
            done[s] = p1
    for (s, n), c in zip(zip(seqs, lens), lm_caches):
        K, V = vals[s]
        c._k[:, :, :n] = synth.bf16_to_f32(K)
        c._v[:, :, :n] = synth.bf16_to_f32(V)
        c.len = n
        assert ctx.seq_len(s) == n
    return vals


def test_kv_write_read_round_trip_is_bit_exact(cuda_ok):
    W, ctx, lm = _model(3, 1024)
    seqs = [ctx.seq_alloc() for _ in range(3)]
    lens = [333, 17, 512]
    caches = [lm.new_cache(n + 4) for n in lens]
    vals = _inject(ctx, caches, seqs, lens, 3, "rt", chunk=40)
    for s, n in zip(seqs, lens):
        K, V = vals[s]
        for l in range(3):
            k, v = ctx.kv_read(s, l, 0, n)
            assert np.array_equal(k, K[l]) and np.array_equal(v, V[l]), (s, l)
            # a window that starts inside a page
            k, v = ctx.kv_read(s, l, 5, n - 9)
            assert np.array_equal(k, K[l, :, 5:n - 4]) and np.array_equal(v, V[l, :, 5:n - 4]), (s, l)
    ctx.close()


@pytest.mark.parametrize("B", [2, 5])
def test_decode_appends_in_place(cuda_ok, B):
    """B = 2: the persistent kernel appends; B = 5: the per-kernel q|k|v
    epilogue does. Old positions stay bit-identical, the new one lands in the
    sequence's own slot with the oracle's value (bf16 tolerance)."""
    layers = 3
    W, ctx, lm = _model(layers, 1024)
    seqs = [ctx.seq_alloc() for _ in range(B)]
    lens = [40 + 37 * i for i in range(B)]  # positions land mid-page and on page starts
    caches = [lm.new_cache(n + 4) for n in lens]
    vals = _inject(ctx, caches, seqs, lens, layers, f"app{B}", chunk=24)
    x = synth.normal_bf16(4, f"append.x.{B}", (B, 896))
    out, _ = ctx.decode(seqs, x)
    for b, (s, n, c) in enumerate(zip(seqs, lens, caches)):
        ro, _ = lm.forward(c, x[b:b + 1])
        d, cs, ok = close(out[b:b + 1], ro)
        assert ok, (b, d, cs)
        assert ctx.seq_len(s) == n + 1
        K, V = vals[s]
        for l in range(layers):
            k, v = ctx.kv_read(s, l, 0, n + 1)
            assert np.array_equal(k[:, :n], K[l]) and np.array_equal(v[:, :n], V[l]), (b, l)
            for got, ref in ((k[:, n], c._k[l, :, n]), (v[:, n], c._v[l, :, n])):
                # the value differs from the oracle's only by f32 summation
                # order and RoPE rounding; a write to another slot would leave
                # this one holding unrelated data (cosine far from 1)
                g = bf(got)
                dd = np.abs(g - ref)
                assert (dd <= 2 * bf16_ulp(ref) + 2e-2).all(), (b, l, dd.max())
                cos = (g * ref).sum(-1) / (np.linalg.norm(g, axis=-1) * np.linalg.norm(ref, axis=-1) + 1e-30)
                assert (cos > 0.999).all(), (b, l, cos)
    ctx.close()


@pytest.mark.parametrize("lens", [[4500], [2100, 4200], [4500, 2100, 300, 3000, 2600]])
def test_attention_over_long_injected_cache(cuda_ok, lens):
    """Decode over caches of 2,100-4,500 positions: one or two rows run the
    persistent kernel (up to 36 chunks of 128 positions, combined by the
    chunk holding the new position); five rows run the per-kernel path,
    whose 18 splits of 256 exceed the 8 a cluster combines, so the split
    kernel writes partials and the combine kernel merges them (config 5's
    2,048-4,096-position contexts take this path)."""
    layers = 2
    B = len(lens)
    W, ctx, lm = _model(layers, 4608)
    seqs = [ctx.seq_alloc() for _ in range(B)]
    caches = [lm.new_cache(n + 4) for n in lens]
    _inject(ctx, caches, seqs, lens, layers, f"long{B}", chunk=512)
    if B <= 4:
        assert ctx.step_kernels(B) == 1  # the persistent kernel serves this batch
    x = synth.normal_bf16(5, f"long.x.{B}", (B, 896))
    for t in range(2):
        out, st = ctx.decode(seqs, x)
        ref = []
        for b in range(B):
            ro, rs = lm.forward(caches[b], x[b:b + 1])
            ref.append(ro[0])
            assert abs(st[b] - rs[0]) < 1e-2
        ref = np.stack(ref)
        d, cs, ok = close(out, ref)
        assert ok, (t, d, cs)
        x = ref
    ctx.close()
