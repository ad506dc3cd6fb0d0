"""GPU parity of the VAE decoder (ming_cuda_vae_decode) against the oracle's
f32 restatement (pinned against HF Qwen2 with a sliding window and torch's
interpolation / ISTFT, tests/test_vae_oracle.py).

The decoder computes in f32 with bf16 weights, as the reference does: the
GPU carries activations as two bf16 parts (~16 significant bits) into f32
tensor-core sums and evaluates the irfft as a product with the DFT basis (also
in two parts), so the waveform is gated relative to its scale: max-abs within
1e-3 of the largest sample and cosine > 0.99999. T = 2, 5 and 24 latents
put 8, 20 and 96 rows through the tiled, staged and tcgen05 linears."""
import numpy as np
import pytest

import ming_b200 as M
import oracle as O
from ming_b200 import synth

pytestmark = pytest.mark.gpu

LAYERS, FF = 2, 1024


@pytest.fixture(scope="module")
def vae(cuda_ok):
    W = synth.vae_weights(seed=3, layers=LAYERS, ff=FF, gains=True)
    cfg = M.default_cfg(layers=0, dit_mode=M.DIT_NONE, agg_blocks=0, vae_layers=LAYERS, vae_ff=FF, vae_window=64,
                        vae_max_latents=64)
    ctx = M.Context(cfg, weights=W)
    yield W, ctx
    ctx.close()


@pytest.mark.parametrize("T", [2, 5, 24])
def test_vae_decode_matches_oracle(vae, T):
    W, ctx = vae
    lat = synth.normal_bf16(4, f"vae.latents.{T}", (T, 64))
    ref = O.vae_decode(W, lat, LAYERS, window=64)
    for _ in range(2):  # the same call twice: bit-identical
        got = ctx.vae_decode(lat)
        assert got.shape == ref.shape == (T * 4 * 882,)
        scale = np.abs(ref).max()
        d = np.abs(got.astype(np.float64) - ref).max()
        cos = float((got.astype(np.float64) * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref)))
        assert d <= 1e-3 * scale and cos > 0.99999, (T, d / scale, cos)
        print(f"vae T={T}: max-abs {d:.3g} ({d / scale:.3g} of the largest sample), cosine {cos:.9f}")
        if _ == 0:
            first = got
        else:
            assert np.array_equal(first, got)


def test_vae_decode_rejects_too_many_latents(vae):
    W, ctx = vae
    with pytest.raises(M.MingError, match="vae_max_latents"):
        ctx.vae_decode(np.zeros((65, 64), np.uint16))


def test_vae_decode_full_size_fragment(cuda_ok):
    """The bench's VAE workload at the real shapes: 24 layers, ff 4864, one
    fragment of 128 latents (512 rows through every linear on the tcgen05
    path), against the oracle under the same gate, and bit-identical on a
    second call."""
    T = 128
    W = synth.vae_weights(seed=2)
    lat = synth.normal_bf16(2, "bench.vae.latents", (T, 64))
    ref = O.vae_decode(W, lat, 24, window=64)
    cfg = M.default_cfg(layers=0, dit_mode=M.DIT_NONE, agg_blocks=0, vae_layers=24, vae_ff=4864, vae_window=64,
                        vae_max_latents=T)
    ctx = M.Context(cfg, weights=W)
    try:
        got = ctx.vae_decode(lat)
        again = ctx.vae_decode(lat)
    finally:
        ctx.close()
    scale = np.abs(ref).max()
    d = np.abs(got.astype(np.float64) - ref).max()
    cos = float((got.astype(np.float64) * ref).sum() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    print(f"vae full size T={T}: max-abs {d:.3g} ({d / scale:.3g} of the largest sample), cosine {cos:.9f}")
    assert got.shape == ref.shape == (T * 4 * 882,)
    assert d <= 1e-3 * scale and cos > 0.99999, (d / scale, cos)
    assert np.array_equal(got, again)
