"""The allocation-free decode step, ming_cuda_lm_decode_noalloc.

It exists for callers that cannot allocate device memory while they decode
(a host real-time audio thread that must not block in cudaMalloc; a process
whose device memory is budgeted by another runtime). It runs the same step as
ming_cuda_lm_decode with its attention scratch in a fixed array compiled into
the library, so its output must match ming_cuda_lm_decode's, and it must keep
matching on a second call, which finds the first call's contents still in the
shared scratch.

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


def _ctx(max_ctx, layers=4):
    W = synth.lm_weights(seed=11, bits=4, layers=layers, qscale=QS)
    cfg = M.default_cfg(layers=layers, weight_bits=4, dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=max_ctx,
                        max_pages=256, max_batch=8, max_seqs=16)
    return M.Context(cfg, weights=W)


def test_noalloc_decode_matches_decode_on_consecutive_calls(cuda_ok):
    ctx = _ctx(512)
    B = 5  # more rows than the persistent kernel serves: both entry points run the per-kernel step
    ref_ids, new_ids = [], []
    for b in range(B):
        p = synth.normal_bf16(11, f"noalloc.prompt.{b}", (20 + 3 * b, 896))
        for ids in (ref_ids, new_ids):
            s = ctx.seq_alloc()
            ctx.prefill(s, p, want_out=False)
            ids.append(s)
    x = synth.normal_bf16(11, "noalloc.x", (B, 896))
    xr = xn = x
    for call in range(2):
        ro, rs = ctx.decode(ref_ids, xr)
        no, ns = ctx.decode_noalloc(new_ids, xn)
        d, c, ok = close(no, ro)
        assert ok, (call, d, c)
        assert np.abs(ns - rs).max() < 1e-2, call
        assert [ctx.seq_len(s) for s in new_ids] == [ctx.seq_len(s) for s in ref_ids]
        xr, xn = ro, no
    ctx.close()


def test_noalloc_decode_rejects_scratch_beyond_its_maximum(cuda_ok):
    # 65536 positions -> 256 attention splits: 5 rows need 4.7 MB of partials,
    # more than the fixed 4 MiB; 4 rows (3.8 MB) fit
    ctx = _ctx(65536, layers=2)
    ids = []
    for b in range(5):
        s = ctx.seq_alloc()
        ctx.prefill(s, synth.normal_bf16(12, f"noalloc.big.{b}", (8, 896)), want_out=False)
        ids.append(s)
    x = synth.normal_bf16(12, "noalloc.big.x", (5, 896))
    with pytest.raises(M.MingError, match="scratch"):
        ctx.decode_noalloc(ids, x)
    assert [ctx.seq_len(s) for s in ids] == [8] * 5  # a rejected call changes nothing
    out, stop = ctx.decode_noalloc(ids[:4], x[:4])
    assert out.shape == (4, 896) and np.isfinite(stop).all()
    ctx.close()
