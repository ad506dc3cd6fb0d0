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


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    return True


def bf(a):
    from ming_b200 import synth
    return synth.bf16_to_f32(a).astype(np.float64)


def close(got, ref, tol=2e-2, min_cos=0.999):
    """The north star's bf16 tolerance: max-abs <= tol and cosine > min_cos per row."""
    g = bf(got).reshape(-1, got.shape[-1]) if got.dtype == np.uint16 else np.asarray(got, np.float64).reshape(-1, got.shape[-1])
    r = bf(ref).reshape(-1, ref.shape[-1]) if ref.dtype == np.uint16 else np.asarray(ref, np.float64).reshape(-1, ref.shape[-1])
    d = np.abs(g - r).max()
    cos = ((g * r).sum(1) / (np.linalg.norm(g, axis=1) * np.linalg.norm(r, axis=1) + 1e-30)).min()
    return d, cos, (d <= tol and cos > min_cos)
