"""Seeded random-init weights and inputs in the reference's tensor layout.

Every tensor is drawn from its own counter-based stream, so a tensor's values
depend only on (seed, name), not on generation order:

  * SplitMix64 (Steele, Lea, Flood 2014): the i-th output of a stream with
    state s0 is mix(s0 + (i+1) * 0x9E3779B97F4A7C15), mix = the SplitMix64
    finaliser; s0 = seed * 0x9E3779B97F4A7C15 ^ FNV-1a-64(name).
  * uniforms u = ((x >> 11) + 1) * 2^-53 in (0, 1];
  * normals by Box-Muller: r = sqrt(-2 ln u1), (r cos 2 pi u2, r sin 2 pi u2);
  * bf16 by round-to-nearest-even of the f32 value.

Names follow src/ming_model.zig (LM, flow head, aggregator); quantized linears
use MLX's QuantizedLinear layout (.weight U32, .scales/.biases BF16).
The benchmark's stated choices: LM weights N(0, 0.02), RMSNorm gains 1; 4-bit codes
uniform 0..15 with scales U(0.005, 0.02) and biases -8*scale (zero-centred,
this build's choice: the benchmark leaves them open). The DiT rotary inv_freq for
random init is 10000^(-2i/64) (the checkpoint buffer is absent here).
"""
import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _fnv1a64(s):
    h = 0xCBF29CE484222325
    for b in s.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _mix(z):
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def stream_u64(seed, name, n, offset=0):
    """n SplitMix64 outputs of the (seed, name) stream starting at `offset`."""
    s0 = np.uint64((seed * 0x9E3779B97F4A7C15 ^ _fnv1a64(name)) & 0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        i = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
        return _mix(s0 + i * GOLDEN)


def uniform(seed, name, n):
    x = stream_u64(seed, name, n)
    return ((x >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)


def normal(seed, name, n):
    m = (n + 1) // 2
    u = uniform(seed, name, 2 * m).reshape(m, 2)
    r = np.sqrt(-2.0 * np.log(u[:, 0]))
    t = 2.0 * np.pi * u[:, 1]
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    return out[:n]


def f32_to_bf16(x):
    """Round-to-nearest-even f32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return u.astype(np.uint16)


def bf16_to_f32(h):
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(seed, name, shape, std=1.0):
    n = int(np.prod(shape))
    # chunked to bound memory for the large LM matrices
    out = np.empty(n, dtype=np.uint16)
    step = 1 << 24
    for o in range(0, n, step):
        k = min(step, n - o)
        v = _normal_at(seed, name, o, k)
        out[o:o + k] = f32_to_bf16((v * std).astype(np.float32))
    return out.reshape(shape)


def _normal_at(seed, name, offset, n):
    # values offset .. offset+n of normal(seed, name, .): pairs are aligned to even offsets
    o0 = offset - (offset & 1)
    m = (n + (offset - o0) + 1) // 2
    x = stream_u64(seed, name, 2 * m, offset=o0)
    u = ((x >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
    u = u.reshape(m, 2)
    r = np.sqrt(-2.0 * np.log(u[:, 0]))
    t = 2.0 * np.pi * u[:, 1]
    out = np.empty(2 * m, dtype=np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    s = offset - o0
    return out[s:s + n]


def ones_bf16(shape):
    return np.full(shape, 0x3F80, dtype=np.uint16)


def quantized(seed, name, out_dim, in_dim, bits=4, group=64, smin=0.005, smax=0.02):
    """MLX affine quantized weight: uniform codes, scales U(smin, smax), biases
    -(2^(bits-1)) * scale. Returns (packed U32 [out, in*bits/32], scales, biases)."""
    per = 32 // bits
    ncode = out_dim * in_dim
    words = stream_u64(seed, name + "#codes", (ncode * bits + 63) // 64)
    # every u64 yields 64/bits codes, little end first
    codes = np.empty(((ncode * bits + 63) // 64) * (64 // bits), dtype=np.uint8)
    mask = np.uint64((1 << bits) - 1)
    for j in range(64 // bits):
        codes[j::64 // bits] = ((words >> np.uint64(bits * j)) & mask).astype(np.uint8)
    codes = codes[:ncode].reshape(out_dim, in_dim)
    packed = pack_codes(codes, bits)
    ng = in_dim // group
    su = uniform(seed, name + "#scales", out_dim * ng)
    scales_f = (smin + (smax - smin) * su).astype(np.float32)
    scales = f32_to_bf16(scales_f).reshape(out_dim, ng)
    biases = f32_to_bf16(-(1 << (bits - 1)) * bf16_to_f32(scales).reshape(-1)).reshape(out_dim, ng)
    return packed, scales, biases


def pack_codes(codes, bits):
    """[rows, cols] uint8 codes -> MLX uint32 words (element j at bits*j)."""
    per = 32 // bits
    r, c = codes.shape
    c4 = codes.reshape(r, c // per, per).astype(np.uint32)
    w = np.zeros((r, c // per), dtype=np.uint32)
    for j in range(per):
        w |= c4[:, :, j] << np.uint32(bits * j)
    return w


def unpack_codes(words, bits, cols):
    per = 32 // bits
    r = words.shape[0]
    out = np.empty((r, cols), dtype=np.uint8)
    mask = np.uint32((1 << bits) - 1)
    for j in range(per):
        out[:, j::per] = ((words >> np.uint32(bits * j)) & mask).astype(np.uint8)
    return out


# ----------------------------------------------------------------------------
# model weight sets
# ----------------------------------------------------------------------------

LM_SHAPE = dict(hidden=896, layers=24, heads=14, kv_heads=2, head_dim=64, ff=4864, theta=1e6, eps=1e-6)


def lm_weights(seed=0, bits=16, layers=24, hidden=896, heads=14, kv_heads=2, ff=4864, std=0.02, group=64,
               qscale=(0.005, 0.02)):
    """Qwen2 LM weights under model.model.* plus the stop head. qscale is the
    U(lo, hi) range of the 4/8-bit group scales (the benchmark's: 0.005..0.02)."""
    W = {}
    H, QD, KD = hidden, heads * 64, kv_heads * 64

    def lin(name, o, i, bias):
        if bits == 16:
            W[name + ".weight"] = normal_bf16(seed, name + ".weight", (o, i), std)
        else:
            q, s, b = quantized(seed, name + ".weight", o, i, bits, group, qscale[0], qscale[1])
            W[name + ".weight"], W[name + ".scales"], W[name + ".biases"] = q, s, b
        if bias:
            W[name + ".bias"] = normal_bf16(seed, name + ".bias", (o,), std)

    for l in range(layers):
        p = f"model.model.layers.{l}"
        W[p + ".input_layernorm.weight"] = ones_bf16((H,))
        W[p + ".post_attention_layernorm.weight"] = ones_bf16((H,))
        lin(p + ".self_attn.q_proj", QD, H, True)
        lin(p + ".self_attn.k_proj", KD, H, True)
        lin(p + ".self_attn.v_proj", KD, H, True)
        lin(p + ".self_attn.o_proj", H, QD, False)
        lin(p + ".mlp.gate_proj", ff, H, False)
        lin(p + ".mlp.up_proj", ff, H, False)
        lin(p + ".mlp.down_proj", H, ff, False)
    W["model.model.norm.weight"] = ones_bf16((H,))
    W["stop_head.weight"] = normal_bf16(seed, "stop_head.weight", (2, H), std)
    W["stop_head.bias"] = normal_bf16(seed, "stop_head.bias", (2,), std)
    return W


def inv_freq(dim=64, base=10000.0):
    return (base ** (-np.arange(0, dim, 2, dtype=np.float64) / dim)).astype(np.float32)


def _dit_blocks(W, seed, prefix, blocks, H, ff, std, adaln):
    for i in range(blocks):
        p = f"{prefix}.blocks.{i}"
        if adaln:
            W[p + ".adaLN_modulation.1.weight"] = normal_bf16(seed, p + ".adaLN_modulation.1.weight", (6 * H, H), std)
            W[p + ".adaLN_modulation.1.bias"] = normal_bf16(seed, p + ".adaLN_modulation.1.bias", (6 * H,), std)
        else:
            W[p + ".norm1.weight"] = ones_bf16((H,))
            W[p + ".norm2.weight"] = ones_bf16((H,))
        for n, o, k in (("attn.to_q", H, H), ("attn.to_k", H, H), ("attn.to_v", H, H), ("attn.to_out.0", H, H),
                        ("mlp.ff.0.0", ff, H), ("mlp.ff.2", H, ff)):
            W[f"{p}.{n}.weight"] = normal_bf16(seed, f"{p}.{n}.weight", (o, k), std)
            W[f"{p}.{n}.bias"] = normal_bf16(seed, f"{p}.{n}.bias", (o,), std)
    W[f"{prefix}.rotary_embed.inv_freq"] = inv_freq()


def _lin(W, seed, name, o, i, std):
    W[name + ".weight"] = normal_bf16(seed, name + ".weight", (o, i), std)
    W[name + ".bias"] = normal_bf16(seed, name + ".bias", (o,), std)


def flow_weights(seed=1, blocks=8, hidden=1024, ff=4096, latent=64, cond=896, freq=256, std=0.02):
    """Reference token-conditioned flow head under flowloss.cfm.model.*."""
    W = {}
    F = "flowloss.cfm.model"
    _dit_blocks(W, seed, F, blocks, hidden, ff, std, False)
    _lin(W, seed, F + ".t_embedder.time_mlp.0", hidden, freq, std)
    _lin(W, seed, F + ".t_embedder.time_mlp.2", hidden, hidden, std)
    _lin(W, seed, F + ".x_embedder", hidden, latent, std)
    _lin(W, seed, F + ".c_embedder.cond_embedder", hidden, cond, std)
    W[F + ".final_layer.norm_final.weight"] = ones_bf16((hidden,))
    _lin(W, seed, F + ".final_layer.linear", latent, hidden, std)
    return W


def agg_weights(seed=1, blocks=8, hidden=1024, ff=4096, latent=64, out=896, std=0.02):
    """Aggregator under linear_proj_audio.*."""
    W = {}
    A = "linear_proj_audio"
    _dit_blocks(W, seed, A, blocks, hidden, ff, std, False)
    _lin(W, seed, A + ".x_embedder", hidden, latent, std)
    W[A + ".word_embedder.weight"] = normal_bf16(seed, A + ".word_embedder.weight", (1, hidden), std)
    W[A + ".final_layer.norm_final.weight"] = ones_bf16((hidden,))
    _lin(W, seed, A + ".final_layer.linear", out, hidden, std)
    return W


def ada_weights(seed=1, blocks=6, hidden=768, ff=3072, latent=64, cond=896, freq=256, std=0.02):
    """The adaLN-Zero head (6 blocks x 768, latent 4 x 64) under adaln_head.*."""
    W = {}
    D = "adaln_head"
    _dit_blocks(W, seed, D, blocks, hidden, ff, std, True)
    _lin(W, seed, D + ".t_embedder.time_mlp.0", hidden, freq, std)
    _lin(W, seed, D + ".t_embedder.time_mlp.2", hidden, hidden, std)
    _lin(W, seed, D + ".x_embedder", hidden, latent, std)
    _lin(W, seed, D + ".c_embedder.cond_embedder", hidden, cond, std)
    _lin(W, seed, D + ".final_layer.adaLN_modulation.1", 2 * hidden, hidden, std)
    _lin(W, seed, D + ".final_layer.linear", latent, hidden, std)
    return W


def latent_proj_weights(seed=1, latent=64, hidden=896, std=0.02):
    """The adaLN head's latent -> next LM input linear (the LM + flow-head
    loop's 64 -> 896 projection) under aggregator.proj."""
    W = {}
    _lin(W, seed, "aggregator.proj", hidden, latent, std)
    return W


def nbytes(weights):
    return sum(v.nbytes for v in weights.values())


_ST_DTYPES = {np.dtype(np.uint16): "BF16", np.dtype(np.uint32): "U32", np.dtype(np.float32): "F32",
              np.dtype(np.float16): "F16", np.dtype(np.int32): "I32", np.dtype(np.int64): "I64"}


def save_safetensors(path, tensors, metadata=None):
    """Writes {name: array} as a safetensors file (uint16 arrays are bf16 bit
    patterns): an 8-byte little-endian header length, the JSON header of
    dtypes, shapes and data offsets, then the tensors' bytes in order."""
    import json
    header, off, blobs = {}, 0, []
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": _ST_DTYPES[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)  # the format pads the header to 8 bytes with spaces
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)


def hann_periodic(n):
    """A periodic Hann window, 0.5 - 0.5 cos(2 pi k / n), f32: the stand-in for
    the checkpoint's audio.decoder.head.istft.window buffer (this build's
    choice for random init)."""
    k = np.arange(n, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2.0 * np.pi * k / n)).astype(np.float32)


def vae_weights(seed=2, layers=24, hidden=896, heads=14, kv_heads=2, ff=4864, latent=64, std=0.02, head_std=0.04,
                gains=False):
    """The VAE decoder under audio.decoder.*: fc1 (latent -> hidden), Qwen2
    layers (decoder.layers.i, decoder.norm), the ISTFT head (head.out, hidden ->
    3530 = log-magnitudes and phases of 1765 bins; head.istft.window). bf16
    weights N(0, std) (head.out N(0, head_std), large enough that the spectra
    vary); RMSNorm gains 1, or U(0.5, 1.5) with gains=True."""
    W = {}
    D = "audio.decoder"
    H, QD, KD = hidden, heads * 64, kv_heads * 64
    _lin(W, seed, D + ".fc1", H, latent, std)
    g = np.random.default_rng(seed)
    for i in range(layers):
        p = f"{D}.decoder.layers.{i}"
        for n in ("input_layernorm", "post_attention_layernorm"):
            W[f"{p}.{n}.weight"] = (f32_to_bf16(g.uniform(0.5, 1.5, H).astype(np.float32)) if gains else ones_bf16((H,)))
        for n, o, k, b in (("self_attn.q_proj", QD, H, True), ("self_attn.k_proj", KD, H, True),
                           ("self_attn.v_proj", KD, H, True), ("self_attn.o_proj", H, QD, False),
                           ("mlp.gate_proj", ff, H, False), ("mlp.up_proj", ff, H, False), ("mlp.down_proj", H, ff, False)):
            W[f"{p}.{n}.weight"] = normal_bf16(seed, f"{p}.{n}.weight", (o, k), std)
            if b:
                W[f"{p}.{n}.bias"] = normal_bf16(seed, f"{p}.{n}.bias", (o,), std)
    W[D + ".decoder.norm.weight"] = ones_bf16((H,))
    _lin(W, seed, D + ".head.out", 3530, H, head_std)
    W[D + ".head.istft.window"] = hann_periodic(3528)
    return W
