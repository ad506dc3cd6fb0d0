"""The allocation-free decode step, ming_cuda_lm_decode_noalloc.

It exists for callers that cannot allocate device memory while they decode
(a host real-time audio thread that must not block in cudaMalloc; a process
whose device memory is budgeted by another runtime). It runs the same step as
ming_cuda_lm_decode with its attention scratch in a fixed array compiled into
the library, so its output must match ming_cuda_lm_decode's, and it must keep
matching on a second call, which finds the first call's contents still in the
shared scratch.

ming_cuda_lm_decode serves up to 4 rows with the persistent decode kernel and
more rows with the per-kernel step; the allocation-free call always runs the
per-kernel step, with the attention splits combined in o_proj's prologue. The
cases below cover both sides of that split, the staged (more than 8 rows) and
tcgen05 (bf16, 64 rows) linears under that prologue, and calls of the two
entry points interleaved on the same sequences.

This file is collected last on purpose: the entry point's scratch is shared by
every call in the process, and the test must pass both alone and after the
other GPU tests have used the library.
"""
import numpy as np
import pytest

import ming_b200 as M
from ming_b200 import synth

from conftest import close

pytestmark = pytest.mark.gpu

QS = (0.002, 0.005)  # the well-conditioned 4-bit scales of the strict LM gates


def _ctx(max_ctx, layers=4, bits=4, max_batch=8, max_seqs=16):
    W = synth.lm_weights(seed=11, bits=bits, layers=layers, qscale=QS)
    cfg = M.default_cfg(layers=layers, weight_bits=bits, dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=max_ctx,
                        max_pages=1024, max_batch=max_batch, max_seqs=max_seqs)
    return M.Context(cfg, weights=W)


def _twin_sequences(ctx, B, tag):
    """Two sets of B sequences with the same prompts (one per entry point)."""
    ref_ids, new_ids = [], []
    for b in range(B):
        p = synth.normal_bf16(11, f"noalloc.{tag}.prompt.{b}", (20 + 3 * (b % 9), 896))
        for ids in (ref_ids, new_ids):
            s = ctx.seq_alloc()
            ctx.prefill(s, p, want_out=False)
            ids.append(s)
    return ref_ids, new_ids


def _compare_consecutive(ctx, B, tag, calls=2):
    ref_ids, new_ids = _twin_sequences(ctx, B, tag)
    x = synth.normal_bf16(11, f"noalloc.{tag}.x", (B, 896))
    xr = xn = x
    for call in range(calls):
        ro, rs = ctx.decode(ref_ids, xr)
        no, ns = ctx.decode_noalloc(new_ids, xn)
        d, c, ok = close(no, ro)
        assert ok, (tag, call, d, c)
        assert np.abs(ns - rs).max() < 1e-2, (tag, call)
        assert [ctx.seq_len(s) for s in new_ids] == [ctx.seq_len(s) for s in ref_ids]
        xr, xn = ro, no
    for s in ref_ids + new_ids:
        ctx.seq_free(s)


@pytest.mark.parametrize("B", [1, 4, 5])
def test_noalloc_decode_matches_decode_on_consecutive_calls(cuda_ok, B):
    # B = 1 and 4: ming_cuda_lm_decode runs the persistent kernel, the
    # allocation-free call the per-kernel step; B = 5: both the per-kernel step
    ctx = _ctx(512)
    _compare_consecutive(ctx, B, f"q4.{B}")
    ctx.close()


@pytest.mark.parametrize("B", [12, 64])
def test_noalloc_decode_bf16_staged_and_tcgen05(cuda_ok, B):
    # bf16 weights: 12 rows take the staged linear (prologue once into
    # fragments), 64 rows the tcgen05 linear, both with the split combine as
    # o_proj's prologue
    ctx = _ctx(256, layers=2, bits=16, max_batch=64, max_seqs=2 * B)
    _compare_consecutive(ctx, B, f"bf16.{B}")
    ctx.close()


def test_noalloc_interleaved_with_decode_on_same_sequences(cuda_ok):
    # the same three sequences stepped alternately by the two entry points
    # track a twin set stepped by ming_cuda_lm_decode only
    ctx = _ctx(512)
    ref_ids, mix_ids = _twin_sequences(ctx, 3, "mix")
    x = synth.normal_bf16(11, "noalloc.mix.x", (3, 896))
    xr = xm = x
    for call in range(4):
        ro, rs = ctx.decode(ref_ids, xr)
        mo, ms = (ctx.decode_noalloc if call % 2 else ctx.decode)(mix_ids, xm)
        d, c, ok = close(mo, ro)
        assert ok, (call, d, c)
        assert np.abs(ms - rs).max() < 1e-2, call
        xr, xm = ro, mo
    ctx.close()


def test_noalloc_decode_rejects_scratch_beyond_its_maximum(cuda_ok):
    # 65536 positions -> 256 attention splits: 5 rows need 4.7 MB of partials,
    # more than the fixed 4 MiB; 4 rows (3.8 MB) fit
    ctx = _ctx(65536, layers=2)
    ids, ref = [], []
    for b in range(5):
        p = synth.normal_bf16(12, f"noalloc.big.{b}", (8, 896))
        for lst in (ids, ref):
            s = ctx.seq_alloc()
            ctx.prefill(s, p, want_out=False)
            lst.append(s)
    x = synth.normal_bf16(12, "noalloc.big.x", (5, 896))
    with pytest.raises(M.MingError, match="scratch"):
        ctx.decode_noalloc(ids, x)
    assert [ctx.seq_len(s) for s in ids] == [8] * 5  # a rejected call changes nothing
    out, stop = ctx.decode_noalloc(ids[:4], x[:4])
    rout, rstop = ctx.decode(ref[:4], x[:4])
    d, c, ok = close(out, rout)
    assert ok, (d, c)
    assert np.abs(stop - rstop).max() < 1e-2
    ctx.close()
