import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "ming-tts-serve_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); runs the CUDA path through the C ABI")


# Gate calls that passed only through within_reference's widening (the strict
# 2e-2 / 0.999 bound failed): listed at the end of the run.
WIDENED = []


def pytest_terminal_summary(terminalreporter):
    if WIDENED:
        terminalreporter.write_line(f"within_reference widened {len(WIDENED)} gate(s) past the strict bound:")
        for w in WIDENED[:40]:
            terminalreporter.write_line("  " + w)


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    return True


def bf(a):
    from ming_b200 import synth
    return synth.bf16_to_f32(a).astype(np.float64)


def bf16_ulp(v):
    """Spacing of bf16 values at |v| (8 significant bits)."""
    a = np.maximum(np.abs(v), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def close(got, ref, tol=2e-2, min_cos=0.999, ulps=2):
    """The north star's bf16 tolerance: every element within max-abs `tol`
    (2e-2) — or, where the reference value is large enough that `ulps` bf16
    rounding steps exceed it (|v| >= 2: one step is 0.0156 in [2, 4), 0.031
    in [4, 8)), within `ulps` steps — and cosine > min_cos per row. Returns
    (max-abs diff, min cosine, ok)."""
    g = bf(got).reshape(-1, got.shape[-1]) if got.dtype == np.uint16 else np.asarray(got, np.float64).reshape(-1, got.shape[-1])
    r = bf(ref).reshape(-1, ref.shape[-1]) if ref.dtype == np.uint16 else np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    diff = np.abs(g - r)
    d = diff.max()
    bound = np.maximum(tol, ulps * bf16_ulp(r))
    cos = ((g * r).sum(1) / (np.linalg.norm(g, axis=1) * np.linalg.norm(r, axis=1) + 1e-30)).min()
    return d, cos, bool((diff <= bound).all() and cos > min_cos)


def within_reference(got, fused, graph, tol=2e-2, min_cos=0.999, ulps=2, exact=None):
    """Parity gate for multi-layer LM outputs against the oracle's fused
    rounding (the reference's fused kernels), scaled by how far the
    reference's own plain graph (oracle GRAPH mode) lies from it on the same
    input. Per row: every element within `close`'s bound (max-abs `tol` or
    `ulps` bf16 steps) or, where the two reference paths already disagree,
    within twice that row's fused-vs-graph max-abs spread; and cosine above
    `min_cos` or above the fused-vs-graph cosine of that row. With `exact`
    (the oracle without bf16 rounding, F32 mode), an element also passes when
    it lies no further from the exact value than the farther of the two
    reference paths plus one bf16 step: no less accurate than the reference
    itself, rounded the other way. Returns (max-abs diff, min cosine, ok)."""
    g, f, r = (bf(a).reshape(-1, a.shape[-1]) for a in (got, fused, graph))
    diff = np.abs(g - f)
    spread = np.abs(r - f).max(1, keepdims=True)
    bound = np.maximum(np.maximum(tol, ulps * bf16_ulp(f)), 2 * spread)
    if exact is not None:
        e = np.asarray(exact, np.float64).reshape(g.shape)
        as_good = np.abs(g - e) <= np.maximum(np.abs(f - e), np.abs(r - e)) + bf16_ulp(e)
        bound = np.where(as_good, np.inf, bound)

    def cos(a, b):
        return (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1) + 1e-30)

    cg, cr = cos(g, f), cos(r, f)
    ok = bool((diff <= bound).all() and (cg > np.minimum(min_cos, cr - 1e-6)).all())
    strict = bool((diff <= np.maximum(tol, ulps * bf16_ulp(f))).all() and (cg > min_cos).all())
    if ok and not strict:
        WIDENED.append(f"{os.environ.get('PYTEST_CURRENT_TEST', '?').split(' ')[0]}: maxabs {diff.max():.4g} cos {cg.min():.6f}")
    return diff.max(), cg.min(), ok


def as_accurate_as_reference(got, fused, graph, exact, rms_ratio=1.5, max_ratio=2.0, cos_slack=1e-4, cos_rel=0.5):
    """Per-row accuracy gate against exact arithmetic (the oracle's F32 mode),
    for outputs where the reference's own two implementations (FUSED kernels,
    GRAPH plain MLX) already differ from each other by more than the strict
    tolerance: the GPU row's RMS and max-abs distance to the exact result
    stay within rms_ratio / max_ratio of the farther reference path's, and
    its cosine error 1 - cos to the exact result within (1 + cos_rel) x
    theirs (the RMS gate's 1.5x), or cos_slack where theirs is tiny: on rows
    whose attention the reference's own paths resolve differently, two
    f32-exact summation orders (the mma.sync and tcgen05 linears) move the
    cosine by ~1e-3 (measured: 0.8856 and 0.8893 against FUSED 0.8891 on
    the flipping row). Returns
    (worst rms ratio, worst max ratio, worst cosine deficit in units of the
    allowed slack, ok)."""
    g, f, r = (bf(a).reshape(-1, a.shape[-1]) for a in (got, fused, graph))
    e = np.asarray(exact, np.float64).reshape(g.shape)

    def rms(a):
        return np.sqrt(((a - e) ** 2).mean(1))

    def cos(a):
        return (a * e).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(e, axis=1) + 1e-30)

    rr = rms(g) / np.maximum(np.maximum(rms(f), rms(r)), 1e-30)
    mr = np.abs(g - e).max(1) / np.maximum(np.maximum(np.abs(f - e).max(1), np.abs(r - e).max(1)), 1e-30)
    cref = np.minimum(cos(f), cos(r))
    cd = (cref - cos(g)) / np.maximum(cos_slack, cos_rel * (1.0 - cref))
    ok = bool((rr <= rms_ratio).all() and (mr <= max_ratio).all() and (cd <= 1.0).all())
    return float(rr.max()), float(mr.max()), float(cd.max()), ok
