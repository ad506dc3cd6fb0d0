"""CPU pins of the oracle's VAE decoder restatement against the golden fixture
(tests/golden/make_golden_vae.py: torch's linear interpolation, Hugging Face
Qwen2 with a sliding window, and a torch restatement of the "same"-padded
ISTFT, all fp32 on the same seeded weights)."""
import os
import sys

import numpy as np

import oracle as O
from ming_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden_vae as G  # noqa: E402

FIX = np.load(os.path.join(HERE, "golden", "vae_ref_f32.npz"))


def _weights():
    return synth.vae_weights(seed=int(FIX["seed"]), layers=int(FIX["layers"]), ff=int(FIX["ff"]))


def test_upsample_matches_torch_interpolate():
    W = _weights()
    lat = synth.normal_bf16(int(FIX["seed"]) + 1, "golden.vae.latents", (int(FIX["T"]), 64))
    up = O.vae_upsample(G.fc1_rows(W, lat))
    assert up.shape == FIX["upsample"].shape
    assert np.abs(up - FIX["upsample"]).max() <= 1e-6 * np.abs(FIX["upsample"]).max()


def test_backbone_matches_hf_qwen2_sliding_window():
    W = _weights()
    out = O.vae_backbone(W, FIX["upsample"], int(FIX["layers"]), window=int(FIX["window"]))
    ref = FIX["backbone"]
    assert np.abs(out - ref).max() <= 2e-5 * np.abs(ref).max(), np.abs(out - ref).max()
    # the window is what makes it the decoder: the full causal mask differs
    full = O.vae_backbone(W, FIX["upsample"], int(FIX["layers"]), window=10 ** 6)
    assert np.abs(full - ref).max() > 1e-2


def test_istft_matches_torch_same_padding():
    F = 4 * int(FIX["T"])
    out = O.vae_istft_w(G.istft_input(F), synth.hann_periodic(3528))
    ref = FIX["istft"]
    assert out.shape == ref.shape == (F * 882,)
    assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max(), np.abs(out - ref).max() / np.abs(ref).max()
