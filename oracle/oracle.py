"""ctypes harness of the CPU oracle (oracle/ming_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm as the checker. Takes the same weight
dictionaries (reference tensor names, numpy arrays) the product library loads.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libming_oracle.so")

MODE_FUSED, MODE_GRAPH, MODE_F32 = 0, 1, 2

U16P = ctypes.POINTER(ctypes.c_uint16)
U32P = ctypes.POINTER(ctypes.c_uint32)
F32P = ctypes.POINTER(ctypes.c_float)


class MoLin(ctypes.Structure):
    _fields_ = [("fmt", ctypes.c_int), ("out", ctypes.c_int), ("in_", ctypes.c_int), ("group", ctypes.c_int),
                ("w", U16P), ("q", U32P), ("scales", U16P), ("biases", U16P), ("bias", U16P)]


class MoLm(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "layers", "heads", "kv_heads", "head_dim", "ff")] + [
        ("theta", ctypes.c_float), ("eps", ctypes.c_float), ("ln1", U16P), ("ln2", U16P),
        ("lin", ctypes.POINTER(MoLin)), ("norm", U16P), ("stop", MoLin)]


class MoKv(ctypes.Structure):
    _fields_ = [("cap", ctypes.c_int), ("len", ctypes.c_int), ("k", F32P), ("v", F32P)]


class MoDit(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "heads", "head_dim", "ff", "blocks")] + [
        ("norm1", U16P), ("norm2", U16P), ("lin", ctypes.POINTER(MoLin)), ("inv_freq", F32P)]


class MoFlow(ctypes.Structure):
    _fields_ = [("dit", MoDit), ("latent", ctypes.c_int), ("cond_dim", ctypes.c_int), ("t_mlp0", MoLin),
                ("t_mlp2", MoLin), ("x_emb", MoLin), ("c_emb", MoLin), ("final_norm", U16P), ("final_lin", MoLin)]


class MoAgg(ctypes.Structure):
    _fields_ = [("dit", MoDit), ("x_emb", MoLin), ("cls", U16P), ("final_norm", U16P), ("final_lin", MoLin)]


class MoAda(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "heads", "head_dim", "ff", "blocks", "latent", "frames",
                                            "cond_dim", "freq_dim")] + [
        ("lin", ctypes.POINTER(MoLin)), ("inv_freq", F32P), ("t_mlp0", MoLin), ("t_mlp2", MoLin), ("x_emb", MoLin),
        ("c_emb", MoLin), ("final_ada", MoLin), ("final_lin", MoLin)]


_lib = None


def build():
    """Compiles the oracle with its Makefile (gcc, OpenMP)."""
    r = subprocess.run(["make", "-s", "-C", HERE], capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.mo_lm_forward.restype = ctypes.c_int
        L.mo_lm_forward_partial.restype = ctypes.c_int
        L.mo_get_threads.restype = ctypes.c_int
        L.mo_bf16_to_f32.restype = ctypes.c_float
        L.mo_bf16_to_f32.argtypes = [ctypes.c_uint16]
        L.mo_f32_to_bf16.restype = ctypes.c_uint16
        L.mo_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib = L
    return _lib


def set_threads(n):
    lib().mo_set_threads(int(n))


def threads():
    return lib().mo_get_threads()


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


class _Keep:
    """Holds numpy arrays alive while ctypes structs point into them."""

    def __init__(self):
        self.refs = []

    def arr(self, a, dtype):
        a = np.ascontiguousarray(a, dtype=dtype)
        self.refs.append(a)
        return a


def make_lin(W, prefix, keep, bias=True):
    w = W[prefix + ".weight"]
    l = MoLin()
    l.group = 64
    if prefix + ".scales" in W:
        sc = keep.arr(W[prefix + ".scales"], np.uint16)
        bi = keep.arr(W[prefix + ".biases"], np.uint16)
        q = keep.arr(w, np.uint32)
        l.out = q.shape[0]
        l.in_ = sc.shape[1] * 64
        l.fmt = q.shape[1] * 32 // l.in_
        l.q, l.scales, l.biases = _p(q, U32P), _p(sc, U16P), _p(bi, U16P)
    else:
        w = keep.arr(w, np.uint16)
        l.fmt, l.out, l.in_ = 16, w.shape[0], w.shape[1]
        l.w = _p(w, U16P)
    if bias and prefix + ".bias" in W:
        l.bias = _p(keep.arr(W[prefix + ".bias"], np.uint16), U16P)
    return l


class Lm:
    """Oracle Qwen2 LM over a weight dict (synth.lm_weights layout)."""

    def __init__(self, W, layers=None, hidden=896, heads=14, kv_heads=2, ff=4864, theta=1e6, eps=1e-6):
        self.keep = _Keep()
        nl = layers if layers is not None else sum(1 for k in W if k.endswith(".input_layernorm.weight"))
        m = MoLm()
        m.hidden, m.layers, m.heads, m.kv_heads, m.head_dim, m.ff = hidden, nl, heads, kv_heads, 64, ff
        m.theta, m.eps = theta, eps
        ln1 = self.keep.arr(np.stack([W[f"model.model.layers.{i}.input_layernorm.weight"] for i in range(nl)]), np.uint16)
        ln2 = self.keep.arr(np.stack([W[f"model.model.layers.{i}.post_attention_layernorm.weight"] for i in range(nl)]),
                            np.uint16)
        lins = (MoLin * (7 * nl))()
        names = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
                 "mlp.up_proj", "mlp.down_proj"]
        for i in range(nl):
            for j, n in enumerate(names):
                lins[i * 7 + j] = make_lin(W, f"model.model.layers.{i}.{n}", self.keep)
        self.lins = lins
        m.ln1, m.ln2, m.lin = _p(ln1, U16P), _p(ln2, U16P), lins
        m.norm = _p(self.keep.arr(W["model.model.norm.weight"], np.uint16), U16P)
        m.stop = make_lin(W, "stop_head", self.keep)
        self.m = m
        self.hidden, self.layers, self.kv_heads = hidden, nl, kv_heads

    def new_cache(self, cap):
        k = np.zeros((self.layers, self.kv_heads, cap, 64), dtype=np.float32)
        v = np.zeros_like(k)
        c = MoKv(cap, 0, _p(k, F32P), _p(v, F32P))
        c._k, c._v = k, v
        return c

    def forward(self, cache, x, mode=MODE_FUSED):
        x = np.ascontiguousarray(x, dtype=np.uint16)
        L = x.shape[0]
        out = np.empty_like(x)
        stop = np.empty(L, dtype=np.float32)
        rc = lib().mo_lm_forward(ctypes.byref(self.m), ctypes.byref(cache), _p(x, U16P), L, _p(out, U16P),
                                 _p(stop, F32P), mode)
        if rc != 0:
            raise RuntimeError("oracle cache overflow")
        return out, stop

    def forward_f32(self, cache, x, mode=MODE_F32):
        x = np.ascontiguousarray(x, dtype=np.uint16)
        out = np.empty(x.shape, dtype=np.float32)
        rc = lib().mo_lm_forward_f32(ctypes.byref(self.m), ctypes.byref(cache), _p(x, U16P), x.shape[0], _p(out, F32P),
                                     mode)
        if rc != 0:
            raise RuntimeError("oracle cache overflow")
        return out

    def forward_partial(self, cache, x, layers_run, mode=MODE_FUSED):
        x = np.ascontiguousarray(x, dtype=np.uint16)
        out = np.empty_like(x)
        rc = lib().mo_lm_forward_partial(ctypes.byref(self.m), ctypes.byref(cache), _p(x, U16P), x.shape[0], layers_run,
                                         _p(out, U16P), mode)
        if rc != 0:
            raise RuntimeError("oracle cache overflow")
        return out


def _dit(W, prefix, blocks, H, ff, keep, adaln=False):
    d = MoDit()
    d.hidden, d.heads, d.head_dim, d.ff, d.blocks = H, H // 64, 64, ff, blocks
    if not adaln:
        d.norm1 = _p(keep.arr(np.stack([W[f"{prefix}.blocks.{i}.norm1.weight"] for i in range(blocks)]), np.uint16), U16P)
        d.norm2 = _p(keep.arr(np.stack([W[f"{prefix}.blocks.{i}.norm2.weight"] for i in range(blocks)]), np.uint16), U16P)
        names = ["attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0", "mlp.ff.0.0", "mlp.ff.2"]
        lins = (MoLin * (6 * blocks))()
        for i in range(blocks):
            for j, n in enumerate(names):
                lins[i * 6 + j] = make_lin(W, f"{prefix}.blocks.{i}.{n}", keep)
        keep.refs.append(lins)
        d.lin = lins
    d.inv_freq = _p(keep.arr(W[f"{prefix}.rotary_embed.inv_freq"], np.float32), F32P)
    return d


class Flow:
    """Oracle token-mode flow head (synth.flow_weights layout)."""

    def __init__(self, W, blocks=8, H=1024, ff=4096, latent=64, cond=896):
        self.keep = _Keep()
        F = "flowloss.cfm.model"
        f = MoFlow()
        f.dit = _dit(W, F, blocks, H, ff, self.keep)
        f.latent, f.cond_dim = latent, cond
        f.t_mlp0 = make_lin(W, F + ".t_embedder.time_mlp.0", self.keep)
        f.t_mlp2 = make_lin(W, F + ".t_embedder.time_mlp.2", self.keep)
        f.x_emb = make_lin(W, F + ".x_embedder", self.keep)
        f.c_emb = make_lin(W, F + ".c_embedder.cond_embedder", self.keep)
        f.final_norm = _p(self.keep.arr(W[F + ".final_layer.norm_final.weight"], np.uint16), U16P)
        f.final_lin = make_lin(W, F + ".final_layer.linear", self.keep)
        self.f, self.H, self.latent = f, H, latent

    def temb(self, mode=MODE_FUSED):
        te = np.empty((10, self.H), dtype=np.uint16)
        lib().mo_flow_temb(ctypes.byref(self.f), _p(te, U16P), mode)
        return te

    def sample(self, z, hist, noise, sde=None, cfg=2.0, shift=0.0, mode=MODE_FUSED):
        z = np.ascontiguousarray(z, dtype=np.uint16)
        hist = np.ascontiguousarray(hist, dtype=np.uint16)
        noise = np.ascontiguousarray(noise, dtype=np.uint16)
        sde = None if sde is None else np.ascontiguousarray(sde, dtype=np.uint16)
        y = np.empty(self.latent, dtype=np.uint16)
        lib().mo_cfm_sample(ctypes.byref(self.f), _p(z, U16P), _p(hist, U16P), _p(noise, U16P), _p(sde, U16P),
                            ctypes.c_float(cfg), ctypes.c_float(shift), _p(y, U16P), mode)
        return y

    def steps(self, z, hist, y, step0, nsteps, sde=None, cfg=2.0, shift=0.0, mode=MODE_FUSED):
        z, hist, y = (np.ascontiguousarray(a, dtype=np.uint16) for a in (z, hist, y))
        sde = None if sde is None else np.ascontiguousarray(sde, dtype=np.uint16)
        out = np.empty(self.latent, dtype=np.uint16)
        lib().mo_cfm_steps(ctypes.byref(self.f), _p(z, U16P), _p(hist, U16P), _p(y, U16P), _p(sde, U16P),
                           ctypes.c_float(cfg), ctypes.c_float(shift), step0, nsteps, _p(out, U16P), mode)
        return out

    def dit_forward(self, x, B, L, mode=MODE_FUSED):
        x = np.ascontiguousarray(x, dtype=np.uint16)
        out = np.empty_like(x)
        lib().mo_dit_forward(ctypes.byref(self.f.dit), _p(x, U16P), B, L, _p(out, U16P), mode)
        return out


class Agg:
    def __init__(self, W, blocks=8, H=1024, ff=4096):
        self.keep = _Keep()
        A = "linear_proj_audio"
        a = MoAgg()
        a.dit = _dit(W, A, blocks, H, ff, self.keep)
        a.x_emb = make_lin(W, A + ".x_embedder", self.keep)
        a.cls = _p(self.keep.arr(W[A + ".word_embedder.weight"].reshape(-1), np.uint16), U16P)
        a.final_norm = _p(self.keep.arr(W[A + ".final_layer.norm_final.weight"], np.uint16), U16P)
        a.final_lin = make_lin(W, A + ".final_layer.linear", self.keep)
        self.a = a
        self.out_dim = a.final_lin.out

    def __call__(self, latent, mode=MODE_FUSED):
        latent = np.ascontiguousarray(latent, dtype=np.uint16)
        B = latent.shape[0]
        out = np.empty((B, self.out_dim), dtype=np.uint16)
        lib().mo_aggregate(ctypes.byref(self.a), _p(latent, U16P), B, _p(out, U16P), mode)
        return out


class Ada:
    """Oracle adaLN head (synth.ada_weights layout)."""

    def __init__(self, W, blocks=6, H=768, ff=3072, latent=64, frames=4, cond=896, freq=256):
        self.keep = _Keep()
        D = "adaln_head"
        a = MoAda()
        a.hidden, a.heads, a.head_dim, a.ff, a.blocks = H, H // 64, 64, ff, blocks
        a.latent, a.frames, a.cond_dim, a.freq_dim = latent, frames, cond, freq
        names = ["adaLN_modulation.1", "attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0", "mlp.ff.0.0", "mlp.ff.2"]
        lins = (MoLin * (7 * blocks))()
        for i in range(blocks):
            for j, n in enumerate(names):
                lins[i * 7 + j] = make_lin(W, f"{D}.blocks.{i}.{n}", self.keep)
        self.lins = lins
        a.lin = lins
        a.inv_freq = _p(self.keep.arr(W[D + ".rotary_embed.inv_freq"], np.float32), F32P)
        a.t_mlp0 = make_lin(W, D + ".t_embedder.time_mlp.0", self.keep)
        a.t_mlp2 = make_lin(W, D + ".t_embedder.time_mlp.2", self.keep)
        a.x_emb = make_lin(W, D + ".x_embedder", self.keep)
        a.c_emb = make_lin(W, D + ".c_embedder.cond_embedder", self.keep)
        a.final_ada = make_lin(W, D + ".final_layer.adaLN_modulation.1", self.keep)
        a.final_lin = make_lin(W, D + ".final_layer.linear", self.keep)
        self.a, self.H, self.latent, self.frames = a, H, latent, frames

    def temb(self, mode=MODE_FUSED):
        te = np.empty((10, self.H), dtype=np.uint16)
        lib().mo_ada_temb(ctypes.byref(self.a), _p(te, U16P), mode)
        return te

    def steps(self, z, y, step0, nsteps, sde=None, cfg=2.0, shift=0.0, mode=MODE_FUSED):
        z = np.ascontiguousarray(z, dtype=np.uint16)
        y = np.ascontiguousarray(y, dtype=np.uint16)
        sde = None if sde is None else np.ascontiguousarray(sde, dtype=np.uint16)
        out = np.empty_like(y)
        lib().mo_ada_steps(ctypes.byref(self.a), z.shape[0], _p(z, U16P), _p(y, U16P), _p(sde, U16P), ctypes.c_float(cfg),
                           ctypes.c_float(shift), step0, nsteps, _p(out, U16P), mode)
        return out

    def sample(self, z, noise, sde=None, cfg=2.0, shift=0.0, mode=MODE_FUSED):
        z = np.ascontiguousarray(z, dtype=np.uint16)
        B = z.shape[0]
        noise = np.ascontiguousarray(noise, dtype=np.uint16)
        sde = None if sde is None else np.ascontiguousarray(sde, dtype=np.uint16)
        y = np.empty_like(noise)
        lib().mo_ada_sample(ctypes.byref(self.a), B, _p(z, U16P), _p(noise, U16P), _p(sde, U16P), ctypes.c_float(cfg),
                            ctypes.c_float(shift), _p(y, U16P), mode)
        return y


def lin_row(W, prefix, row, keep=None):
    """Dequantized weight row (f32) via the oracle's MLX-affine formula."""
    keep = keep or _Keep()
    l = make_lin(W, prefix, keep, bias=False)
    out = np.empty(l.in_, dtype=np.float32)
    lib().mo_lin_row(ctypes.byref(l), row, _p(out, F32P))
    return out


def lin_dequant(W, prefix):
    keep = _Keep()
    l = make_lin(W, prefix, keep, bias=False)
    out = np.empty((l.out, l.in_), dtype=np.float32)
    lib().mo_lin_dequant(ctypes.byref(l), _p(out, F32P))
    return out


def unpack(words, rows, cols, bits):
    words = np.ascontiguousarray(words, dtype=np.uint32)
    codes = np.empty((rows, cols), dtype=np.uint8)
    lib().mo_unpack(_p(words, U32P), rows, cols, bits, codes.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    return codes


def pack(codes, bits):
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    rows, cols = codes.shape
    words = np.empty((rows, cols * bits // 32), dtype=np.uint32)
    lib().mo_pack(codes.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), rows, cols, bits, _p(words, U32P))
    return words


def ada_latent_proj(W, latent):
    """The adaLN head's latent path into the next LM input (the LM + flow-head
    loop's 64 -> 896 linear; no reference code, choice pinned with the product):
    the mean of the patch's frames in f32, frames in order, rounded to bf16;
    then aggregator.proj as an f32 dot plus bias, rounded to bf16.
    latent: uint16 bf16 [B][F][64] -> uint16 [B][896]."""
    def f32(h):
        return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)

    def bf(x):
        u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    lat = f32(latent)
    s = np.zeros(lat.shape[::2], np.float32)
    for f in range(lat.shape[1]):
        s = s + lat[:, f, :]
    m = f32(bf(s / np.float32(lat.shape[1])))
    w = f32(W["aggregator.proj.weight"]).astype(np.float64)
    b = f32(W["aggregator.proj.bias"]).astype(np.float64)
    return bf((m.astype(np.float64) @ w.T + b).astype(np.float32))


# ---------------------------------------------------------------------------
# VAE decoder (numpy restatement; test infrastructure like the rest of this
# module). Follows Model.vaeDecode (src/ming_model.zig:1257-1300),
# linearUpsample (:1303-1342) and QStack.forward with a sliding window
# (:566-614, slidingMask :617-635): the backbone in f32 (MLX promotes the bf16
# weights), fc1 in bf16 (the latents' dtype).
# ---------------------------------------------------------------------------

VAE_HOP, VAE_NFFT, VAE_PATCH = 882, 3528, 4


def _f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _bf16_round(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def vae_upsample(x, scale=VAE_PATCH):
    """Decoder._linear_upsample_1d (align_corners=False) in f32 over rows of x [T][C]:
    row i reads source position p = (i + 0.5) / scale - 0.5 (src/ming_model.zig:1303-1342)."""
    x = np.asarray(x, np.float32)
    T = x.shape[0]
    i = np.arange(T * scale, dtype=np.float32)
    p = (i + np.float32(0.5)) / np.float32(scale) - np.float32(0.5)
    lf = np.floor(p)
    w = (p - lf).astype(np.float32)
    l = lf.astype(np.int64)
    a, b = np.clip(l, 0, T - 1), np.clip(l + 1, 0, T - 1)
    return (x[a] * (np.float32(1) - w)[:, None] + x[b] * w[:, None]).astype(np.float32)


def vae_istft_w(p, win):
    """The ISTFT head on the head's output p [F][3530] with the window win [3528]
    (src/ming_model.zig:1262-1299): magnitude min(exp(m), 100), phase, irfft of
    3528 points ("backward" norm), the window, overlap-add at hop 882 (frame
    parts in the reference's order), the window envelope and the "same" trim
    of (3528 - 882) / 2 samples per side."""
    p = np.asarray(p, np.float32)
    nb = VAE_NFFT // 2 + 1
    mag = np.minimum(np.exp(p[:, :nb]), np.float32(100.0))
    ph = p[:, nb:]
    spec = mag.astype(np.complex64) * (np.cos(ph) + 1j * np.sin(ph)).astype(np.complex64)
    frames = np.fft.irfft(spec, n=VAE_NFFT, axis=-1).astype(np.float32) * np.asarray(win, np.float32)[None, :]
    F = frames.shape[0]
    total = (F + 3) * VAE_HOP
    out = np.zeros(total, np.float32)
    parts = frames.reshape(F, 4, VAE_HOP)
    for j in (3, 2, 1, 0):  # part j of frame t lands in hop block t + j; added j = 3 first
        out[j * VAE_HOP:(j + F) * VAE_HOP] += parts[:, j, :].reshape(-1)
    env = np.zeros(total, np.float32)
    w2 = (np.asarray(win, np.float32) * np.asarray(win, np.float32))
    for t in range(F):
        env[t * VAE_HOP:t * VAE_HOP + VAE_NFFT] += w2
    pad = (VAE_NFFT - VAE_HOP) // 2
    n_out = total - 2 * pad
    return (out[pad:pad + n_out] / np.maximum(env[pad:pad + n_out], np.float32(1e-11))).astype(np.float32)


def vae_decode(W, latents, layers, window=64, heads=14, kv_heads=2, eps=1e-6, theta=1e6):
    """latents uint16 bf16 [T][64] -> waveform f32 [T * 4 * 882]."""
    D = "audio.decoder"
    lat = _f32(latents)
    x = _bf16_round(lat @ _f32(W[D + ".fc1.weight"]).T + _f32(W[D + ".fc1.bias"]))
    xn = vae_backbone(W, vae_upsample(x), layers, window, heads, kv_heads, eps, theta)
    pr = xn @ _f32(W[D + ".head.out.weight"]).T + _f32(W[D + ".head.out.bias"])
    return vae_istft_w(pr, W[D + ".head.istft.window"])


def vae_backbone(W, x, layers, window=64, heads=14, kv_heads=2, eps=1e-6, theta=1e6):
    """The decoder's Qwen2 layers in f32 over upsampled rows x [F][H] with the
    causal sliding window, then the final norm (QStack.forward,
    src/ming_model.zig:566-614)."""
    D = "audio.decoder"
    x = np.asarray(x, np.float32)
    F, H = x.shape
    hd = 64
    half = hd // 2
    l2t = np.float32(np.log2(np.float32(theta)))
    inv_freq = np.exp2(-(np.arange(half, dtype=np.float32) / np.float32(half)) * l2t).astype(np.float32)
    ang = np.arange(F, dtype=np.float32)[:, None] * inv_freq[None, :]
    cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)

    def rms(v, g):
        inv = (np.float32(1) / np.sqrt((v * v).mean(-1, keepdims=True, dtype=np.float32) + np.float32(eps))).astype(np.float32)
        return (v * inv) * _f32(g)[None, :]

    def lin(v, name, bias=False):
        y = v @ _f32(W[name + ".weight"]).T
        return (y + _f32(W[name + ".bias"])) if bias else y

    def rope(t):
        t = t.reshape(F, -1, hd)
        a, b = t[..., :half], t[..., half:]
        c, s = cs[:, None, :], sn[:, None, :]
        return np.concatenate([a * c - b * s, a * s + b * c], -1)

    idx = np.arange(F)
    mask = np.where((idx[None, :] > idx[:, None] - window) & (idx[:, None] >= idx[None, :]), np.float32(0),
                    np.float32(-3.4028235e38)).astype(np.float32)
    grp = heads // kv_heads
    for l in range(layers):
        p = f"{D}.decoder.layers.{l}"
        h = rms(x, W[p + ".input_layernorm.weight"])
        q = rope(lin(h, p + ".self_attn.q_proj", True))
        k = rope(lin(h, p + ".self_attn.k_proj", True))
        v = lin(h, p + ".self_attn.v_proj", True).reshape(F, kv_heads, hd)
        o = np.empty((F, heads, hd), np.float32)
        for hh in range(heads):
            g = hh // grp
            sc = (q[:, hh, :] @ k[:, g, :].T) * np.float32(1.0 / 8.0) + mask
            sc = sc - sc.max(-1, keepdims=True)
            e = np.exp(sc)
            o[:, hh, :] = (e / e.sum(-1, keepdims=True)) @ v[:, g, :]
        x = x + lin(o.reshape(F, heads * hd), p + ".self_attn.o_proj")
        h2 = rms(x, W[p + ".post_attention_layernorm.weight"])
        gt, up = lin(h2, p + ".mlp.gate_proj"), lin(h2, p + ".mlp.up_proj")
        x = x + lin((gt * (np.float32(1) / (np.float32(1) + np.exp(-gt)))) * up, p + ".mlp.down_proj")
    return rms(x, W[D + ".decoder.norm.weight"]).astype(np.float32)
