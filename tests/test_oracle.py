"""CPU tests of the oracle (the checker): pinned against Hugging Face Qwen2
fp32 fixtures, MLX-packing known answers, and independent numpy restatements
of the DiT / CFM math (F32 mode)."""
import numpy as np
import pytest

import oracle as O
from ming_b200 import synth

from conftest import bf


def test_oracle_lm_matches_hf_qwen2_f32():
    from make_golden import lm_inputs
    g = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "lm_hf_f32.npz"))
    W = synth.lm_weights(seed=int(g["seed"]), bits=16, layers=int(g["layers"]))
    lm = O.Lm(W)
    x = lm_inputs()
    P, D = int(g["prefill"]), int(g["decode"])
    c = lm.new_cache(64)
    outs = [lm.forward_f32(c, x[:P])]
    for i in range(D):
        outs.append(lm.forward_f32(c, x[P + i:P + i + 1]))
    h = np.concatenate(outs)
    assert np.abs(h - g["hidden"]).max() < 2e-5 * max(1.0, np.abs(g["hidden"]).max())
    # the bf16 rounding modes stay within bf16 noise of the fp32 model
    for mode in (O.MODE_FUSED, O.MODE_GRAPH):
        c = lm.new_cache(64)
        outs = [lm.forward(c, x[:P], mode)[0]] + [lm.forward(c, x[P + i:P + i + 1], mode)[0] for i in range(D)]
        hb = bf(np.concatenate(outs))
        cos = (hb * g["hidden"]).sum(1) / np.linalg.norm(hb, axis=1) / np.linalg.norm(g["hidden"], axis=1)
        assert cos.min() > 0.9999


def test_mlx_pack_known_answers():
    # 4-bit: element j of a word at bits 4j, little end first
    codes = np.array([[0, 1, 2, 3, 4, 5, 6, 7, 15, 14, 13, 12, 11, 10, 9, 8]], dtype=np.uint8)
    w = O.pack(codes, 4)
    assert w.tolist() == [[0x76543210, 0x89ABCDEF]]
    assert (O.unpack(w, 1, 16, 4) == codes).all()
    # 8-bit: element j at bits 8j
    codes8 = np.array([[1, 2, 3, 4, 0xFF, 0, 0x80, 0x7F]], dtype=np.uint8)
    w8 = O.pack(codes8, 8)
    assert w8.tolist() == [[0x04030201, 0x7F8000FF]]
    assert (O.unpack(w8, 1, 8, 8) == codes8).all()
    # the synth packer and the oracle agree bit for bit
    rng = np.random.default_rng(0)
    for bits in (4, 8):
        c = rng.integers(0, 1 << bits, size=(7, 128), dtype=np.uint8)
        assert (synth.pack_codes(c, bits) == O.pack(c, bits)).all()
        assert (synth.unpack_codes(O.pack(c, bits), bits, 128) == c).all()


def test_dequant_is_mlx_affine():
    for bits in (4, 8):
        q, s, b = synth.quantized(3, "t.weight", 5, 192, bits)
        W = {"t.weight": q, "t.scales": s, "t.biases": b}
        codes = synth.unpack_codes(q, bits, 192).astype(np.float32)
        sf = np.repeat(synth.bf16_to_f32(s), 64, axis=1)
        bfv = np.repeat(synth.bf16_to_f32(b), 64, axis=1)
        ref = (sf * codes + bfv).astype(np.float32)
        for r in range(5):
            assert (O.lin_row(W, "t", r) == ref[r]).all()
        # the benchmark's distribution: codes uniform over 0..2^bits-1, scales in [0.005, 0.02]
        assert codes.max() == (1 << bits) - 1 and codes.min() == 0
        assert 0.0049 <= synth.bf16_to_f32(s).min() and synth.bf16_to_f32(s).max() <= 0.0201


def test_synth_is_counter_based():
    a = synth.normal_bf16(5, "x", (1000,))
    b = synth.normal_bf16(5, "x", (2000,))[:1000]
    assert (a == b).all()
    assert not (synth.normal_bf16(6, "x", (1000,)) == a).all()
    v = synth.bf16_to_f32(synth.normal_bf16(0, "stats", (200000,)))
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1) < 0.01


def _rb(x):
    return synth.bf16_to_f32(synth.f32_to_bf16(np.asarray(x, dtype=np.float32)))


def test_flow_schedule_bf16():
    t = np.empty(11, np.float32)
    dt = np.empty(10, np.float32)
    sq = np.empty(10, np.float32)
    P = lambda a: a.ctypes.data_as(O.F32P)
    O.lib().mo_flow_schedule(P(t), P(dt), P(sq))
    s = _rb(np.array([0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32], np.float32))
    tt = _rb(_rb(1 / 32) * s)
    ct = _rb(np.cos(_rb(_rb(np.pi / 2) * tt)))
    ref = _rb(tt - _rb(_rb(ct - 1) + tt))
    assert np.allclose(t, ref, atol=0, rtol=0)
    assert t[0] == 0 and abs(t[-1] - 1) < 1e-2
    assert np.array_equal(dt, _rb(ref[1:] - ref[:-1]))


# ---- independent numpy restatements in F32 mode (no rounding) ----

def _lin(W, p, x):
    w = synth.bf16_to_f32(W[p + ".weight"]).astype(np.float64)
    y = x @ w.T
    if p + ".bias" in W:
        y = y + synth.bf16_to_f32(W[p + ".bias"])
    return y


def _rotary(x, pos, invf):
    ang = pos[:, None] * invf[None, :]
    c, s = np.cos(ang), np.sin(ang)
    xr = x.reshape(x.shape[0], -1, 32, 2)
    e, o = xr[..., 0], xr[..., 1]
    out = np.stack([e * c[:, None] - o * s[:, None], e * s[:, None] + o * c[:, None]], -1)
    return out.reshape(x.shape)


def _attn(q, k, v, B, L, heads):
    q = q.reshape(B, L, heads, 64)
    k = k.reshape(B, L, heads, 64)
    v = v.reshape(B, L, heads, 64)
    s = np.einsum("blhd,bmhd->bhlm", q / 8, k)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.einsum("bhlm,bmhd->blhd", p, v).reshape(B * L, heads * 64)


def _gelu(x):
    return 0.5 * x * (1 + np.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def _rms(x, eps=1e-6):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)


def _ln(x, eps=1e-6):
    m = x.mean(-1, keepdims=True)
    return (x - m) / np.sqrt(((x - m) ** 2).mean(-1, keepdims=True) + eps)


def test_oracle_dit_token_matches_numpy_f32():
    H, FF, NB, B, L = 128, 256, 2, 2, 3
    W = synth.flow_weights(seed=4, blocks=NB, hidden=H, ff=FF, std=0.05)
    f = O.Flow(W, blocks=NB, H=H, ff=FF)
    x = synth.normal_bf16(9, "dit.x", (B * L, H))
    got = bf(f.dit_forward(x, B, L, O.MODE_F32))
    xs = bf(x)
    invf = W["flowloss.cfm.model.rotary_embed.inv_freq"].astype(np.float64)
    pos = np.tile(np.arange(L), B).astype(np.float64)
    for i in range(NB):
        p = f"flowloss.cfm.model.blocks.{i}"
        h = _rms(xs)
        q = _rotary(_lin(W, p + ".attn.to_q", h), pos, invf)
        k = _rotary(_lin(W, p + ".attn.to_k", h), pos, invf)
        v = _lin(W, p + ".attn.to_v", h)
        xs = xs + _lin(W, p + ".attn.to_out.0", _attn(q, k, v, B, L, H // 64))
        xs = xs + _lin(W, p + ".mlp.ff.2", _gelu(_lin(W, p + ".mlp.ff.0.0", _rms(xs))))
    # the oracle's output is stored in bf16
    assert np.abs(got - xs).max() <= 2 ** -8 * np.abs(xs).max() + 1e-6


def _temb_np(W, pre, t, freq=256):
    half = freq // 2
    e = np.float32(np.log(10000.0) / (half - 1))
    f = np.exp(np.arange(half, dtype=np.float32) * -e).astype(np.float64)
    a = (1000.0 * t)[:, None] * f[None, :]
    sc = np.concatenate([np.sin(a), np.cos(a)], -1)
    h = _lin(W, pre + ".t_embedder.time_mlp.0", sc)
    h = h / (1 + np.exp(-h))
    return _lin(W, pre + ".t_embedder.time_mlp.2", h)


def _sched_f32():
    s = np.array([0, 2, 4, 6, 8, 12, 16, 20, 24, 28, 32], np.float64) / 32
    return s - (np.cos(np.pi / 2 * s) - 1 + s)


def test_oracle_cfm_token_matches_numpy_f32():
    H, FF, NB, LAT, CD = 128, 256, 2, 64, 896
    W = synth.flow_weights(seed=5, blocks=NB, hidden=H, ff=FF, std=0.05)
    f = O.Flow(W, blocks=NB, H=H, ff=FF)
    z = synth.normal_bf16(1, "cfm.z", (CD,))
    hist = synth.normal_bf16(1, "cfm.hist", (LAT,))
    noise = synth.normal_bf16(1, "cfm.noise", (LAT,))
    got = bf(f.sample(z, hist, noise, None, 2.0, 0.0, O.MODE_F32))
    F = "flowloss.cfm.model"
    t = _sched_f32()
    te = _temb_np(W, F, t[:10])
    ce = np.stack([_lin(W, F + ".c_embedder.cond_embedder", bf(z)), _lin(W, F + ".c_embedder.cond_embedder", np.zeros(CD))])
    xh = _lin(W, F + ".x_embedder", bf(hist))
    y = bf(noise)
    invf = W[F + ".rotary_embed.inv_freq"].astype(np.float64)
    pos = np.tile(np.arange(3), 2).astype(np.float64)
    for s in range(10):
        xe = _lin(W, F + ".x_embedder", y)
        rows = np.stack([te[s] + ce[0], xh, xe, te[s] + ce[1], xh, xe])
        for i in range(NB):
            p = f"{F}.blocks.{i}"
            h = _rms(rows)
            q = _rotary(_lin(W, p + ".attn.to_q", h), pos, invf)
            k = _rotary(_lin(W, p + ".attn.to_k", h), pos, invf)
            v = _lin(W, p + ".attn.to_v", h)
            rows = rows + _lin(W, p + ".attn.to_out.0", _attn(q, k, v, 2, 3, H // 64))
            rows = rows + _lin(W, p + ".mlp.ff.2", _gelu(_lin(W, p + ".mlp.ff.0.0", _rms(rows))))
        out = _lin(W, F + ".final_layer.linear", _rms(rows[[2, 5]]))
        fvel = out[0] + (out[0] - out[1]) * 2.0
        y = y + (t[s + 1] - t[s]) * fvel
    assert np.abs(got - y).max() <= 2 ** -7 * max(1.0, np.abs(y).max())


def test_oracle_ada_matches_numpy_f32():
    H, FF, NB, LAT, CD, Fr, B = 128, 256, 2, 64, 896, 4, 2
    W = synth.ada_weights(seed=6, blocks=NB, hidden=H, ff=FF, std=0.05)
    a = O.Ada(W, blocks=NB, H=H, ff=FF, frames=Fr)
    z = synth.normal_bf16(2, "ada.z", (B, CD))
    noise = synth.normal_bf16(2, "ada.noise", (B, Fr, LAT))
    got = bf(a.sample(z, noise, None, 2.0, 0.0, O.MODE_F32))
    D = "adaln_head"
    t = _sched_f32()
    te = _temb_np(W, D, t[:10])
    zc = np.concatenate([bf(z), np.zeros((B, CD))])
    ce = _lin(W, D + ".c_embedder.cond_embedder", zc)
    y = bf(noise).reshape(B, Fr, LAT)
    invf = W[D + ".rotary_embed.inv_freq"].astype(np.float64)
    pos = np.tile(np.arange(Fr), 2 * B).astype(np.float64)
    for s in range(10):
        c = te[s] + ce
        sc = c / (1 + np.exp(-c))
        x = _lin(W, D + ".x_embedder", np.concatenate([y, y]).reshape(2 * B * Fr, LAT))
        for i in range(NB):
            p = f"{D}.blocks.{i}"
            m = np.repeat(_lin(W, p + ".adaLN_modulation.1", sc), Fr, axis=0)
            sh1, s1, g1, sh2, s2, g2 = np.split(m, 6, axis=1)
            h = _ln(x) * (1 + s1) + sh1
            q = _rotary(_lin(W, p + ".attn.to_q", h), pos, invf)
            k = _rotary(_lin(W, p + ".attn.to_k", h), pos, invf)
            v = _lin(W, p + ".attn.to_v", h)
            x = x + g1 * _lin(W, p + ".attn.to_out.0", _attn(q, k, v, 2 * B, Fr, H // 64))
            h = _ln(x) * (1 + s2) + sh2
            x = x + g2 * _lin(W, p + ".mlp.ff.2", _gelu(_lin(W, p + ".mlp.ff.0.0", h)))
        fm = np.repeat(_lin(W, D + ".final_layer.adaLN_modulation.1", sc), Fr, axis=0)
        shf, sf = np.split(fm, 2, axis=1)
        vel = _lin(W, D + ".final_layer.linear", _ln(x) * (1 + sf) + shf).reshape(2, B, Fr, LAT)
        y = y + (t[s + 1] - t[s]) * (vel[0] + (vel[0] - vel[1]) * 2.0)
    assert np.abs(got - y.reshape(got.shape)).max() <= 2 ** -7 * max(1.0, np.abs(y).max())
