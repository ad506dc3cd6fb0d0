"""Python binding of libming_cuda.so (include/ming_cuda.h) — the B200 hot path
of ming-tts-serve: the Qwen2 LM decode step and the DiT flow head.

This is a thin ctypes mirror of the C ABI, the same calls a Zig host makes
through `extern` declarations. The library must have been built
(ming-tts-serve_b200/build.py); there is no CPU fallback: every compute call
raises if the CUDA library is missing or fails.
"""
import ctypes
import os

import numpy as np

from . import synth  # noqa: F401

HERE = os.path.dirname(os.path.abspath(__file__))
# MING_CUDA_LIB selects another build of the library (e.g. one compiled with
# different tuning constants) for side-by-side timing; default: the in-tree build
LIB_PATH = os.environ.get("MING_CUDA_LIB") or os.path.join(os.path.dirname(HERE), "libming_cuda.so")

MING_OK = 0
DTYPE_BF16, DTYPE_F32, DTYPE_U32 = 0, 1, 2
PTR_HOST, PTR_DEVICE = 0, 1
DIT_NONE, DIT_TOKEN, DIT_ADALN = 0, 1, 2

# Exported symbols, in header order (tests check the library exports each).
SYMBOLS = [
    "ming_cuda_default_cfg", "ming_cuda_create", "ming_cuda_load_tensor", "ming_cuda_finalize",
    "ming_cuda_seq_alloc", "ming_cuda_seq_free", "ming_cuda_seq_len", "ming_cuda_seq_truncate",
    "ming_cuda_lm_prefill", "ming_cuda_lm_decode", "ming_cuda_lm_generate", "ming_cuda_cfm_sample",
    "ming_cuda_cfm_steps",
    "ming_cuda_aggregate", "ming_cuda_get_stream", "ming_cuda_sync", "ming_cuda_destroy",
    "ming_cuda_last_error", "ming_cuda_kv_read", "ming_cuda_unpack_linear", "ming_cuda_flow_temb",
    "ming_cuda_step_kernels", "ming_cuda_lm_decode_noalloc", "ming_cuda_kv_write",
    "ming_cuda_default_sample_params", "ming_cuda_sample_latents", "ming_cuda_loop_create", "ming_cuda_loop_submit",
    "ming_cuda_loop_step", "ming_cuda_loop_result", "ming_cuda_loop_destroy", "ming_cuda_load_safetensors",
    "ming_cuda_vae_decode",
]


class Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "layers", "heads", "kv_heads", "head_dim", "ff")] + [
        ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float)] + [
        (n, ctypes.c_int) for n in (
            "weight_bits", "group_size", "page_size", "max_seqs", "max_pages", "max_ctx", "max_batch", "max_prefill",
            "dit_mode", "dit_hidden", "dit_blocks", "dit_heads", "dit_ff", "dit_latent", "dit_frames",
            "dit_cond_dim", "dit_freq_dim", "dit_max_batch", "agg_blocks", "vae_layers", "vae_ff", "vae_window",
            "vae_max_latents")]


class SampleParams(ctypes.Structure):
    """ming_sample_params: SampleParams (src/ming_model.zig:1368-1373) + max_len."""
    _fields_ = [("max_steps", ctypes.c_int), ("max_len", ctypes.c_int), ("cfg", ctypes.c_float),
                ("sigma", ctypes.c_float), ("temperature", ctypes.c_float)]


class MingError(RuntimeError):
    pass


_lib = None


def lib():
    """Loads libming_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise MingError(f"{LIB_PATH} is missing: build it with ming-tts-serve_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    IP = ctypes.POINTER(ctypes.c_int)
    sig = {
        "ming_cuda_default_cfg": (None, [ctypes.POINTER(Cfg)]),
        "ming_cuda_create": (I, [I, ctypes.POINTER(Cfg), ctypes.POINTER(P)]),
        "ming_cuda_load_tensor": (I, [P, ctypes.c_char_p, I, ctypes.POINTER(ctypes.c_int64), I, P]),
        "ming_cuda_finalize": (I, [P]),
        "ming_cuda_seq_alloc": (I, [P, IP]),
        "ming_cuda_seq_free": (I, [P, I]),
        "ming_cuda_seq_len": (I, [P, I, IP]),
        "ming_cuda_seq_truncate": (I, [P, I, I]),
        "ming_cuda_lm_prefill": (I, [P, I, P, I, P, P, I]),
        "ming_cuda_lm_decode": (I, [P, I, IP, P, P, P, I]),
        "ming_cuda_lm_generate": (I, [P, I, IP, P, I, P, P, I]),
        "ming_cuda_cfm_sample": (I, [P, I, P, P, P, P, F, F, P, I]),
        "ming_cuda_cfm_steps": (I, [P, I, P, P, P, P, F, F, I, I, P, I]),
        "ming_cuda_aggregate": (I, [P, I, P, P, I]),
        "ming_cuda_get_stream": (I, [P, ctypes.POINTER(P)]),
        "ming_cuda_sync": (I, [P]),
        "ming_cuda_destroy": (I, [P]),
        "ming_cuda_last_error": (ctypes.c_char_p, []),
        "ming_cuda_kv_read": (I, [P, I, I, I, I, P, P]),
        "ming_cuda_kv_write": (I, [P, I, I, I, I, P, P]),
        "ming_cuda_unpack_linear": (I, [P, ctypes.c_char_p, P]),
        "ming_cuda_flow_temb": (I, [P, P]),
        "ming_cuda_default_sample_params": (None, [ctypes.POINTER(SampleParams)]),
        "ming_cuda_sample_latents": (I, [P, P, I, P, ctypes.POINTER(SampleParams), P, I, ctypes.c_uint64, P, I, IP, P,
                                         P]),
        "ming_cuda_loop_create": (I, [P, I, ctypes.POINTER(SampleParams), ctypes.POINTER(P)]),
        "ming_cuda_loop_submit": (I, [P, P, I, P, P, I, ctypes.c_uint64, I, IP]),
        "ming_cuda_loop_step": (I, [P, IP, IP]),
        "ming_cuda_loop_result": (I, [P, I, P, I, IP, P, P]),
        "ming_cuda_loop_destroy": (I, [P]),
        "ming_cuda_load_safetensors": (I, [P, ctypes.c_char_p, IP]),
        "ming_cuda_vae_decode": (I, [P, P, I, P, I]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _check(rc):
    if rc != MING_OK:
        msg = lib().ming_cuda_last_error().decode(errors="replace")
        raise MingError(f"ming_cuda error {rc}: {msg}")


def default_cfg(**kw):
    c = Cfg()
    lib().ming_cuda_default_cfg(ctypes.byref(c))
    for k, v in kw.items():
        if not hasattr(c, k):
            raise KeyError(k)
        setattr(c, k, v)
    return c


def sample_params(**kw):
    """Default sampling parameters (max_steps 1000, max_len 512, cfg 2.0,
    sigma 0.25, temperature 0.0) with overrides."""
    p = SampleParams()
    lib().ming_cuda_default_sample_params(ctypes.byref(p))
    for k, v in kw.items():
        if not hasattr(p, k):
            raise KeyError(k)
        setattr(p, k, v)
    return p


def check_safetensors(path):
    """Validates a safetensors checkpoint without a context (no GPU needed);
    returns how many hot-path tensors it would load."""
    n = ctypes.c_int(0)
    _check(lib().ming_cuda_load_safetensors(None, os.fsencode(path), ctypes.byref(n)))
    return n.value


def _ptr(a):
    """Host numpy array -> void*; device tensor (has data_ptr) -> its address."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return ctypes.c_void_p(a.data_ptr())
    assert a.flags["C_CONTIGUOUS"], "arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _dtype_code(a):
    if a.dtype == np.uint16:
        return DTYPE_BF16
    if a.dtype == np.float32:
        return DTYPE_F32
    if a.dtype == np.uint32:
        return DTYPE_U32
    raise TypeError(f"unsupported dtype {a.dtype}")


class Context:
    """One device context (ming_ctx). Mirrors the reference Model's hot-path
    surface: load, lm_prefill/lm_decode (lmForward), generate (the token loop),
    cfm_sample (cfmSample), aggregate."""

    def __init__(self, cfg=None, device=0, weights=None, checkpoint=None):
        """weights: {name: array} loaded tensor by tensor; checkpoint: a
        safetensors file (or a directory holding model.safetensors)."""
        self.cfg = cfg if cfg is not None else default_cfg()
        self._h = ctypes.c_void_p()
        _check(lib().ming_cuda_create(device, ctypes.byref(self.cfg), ctypes.byref(self._h)))
        if checkpoint is not None:
            self.load_safetensors(checkpoint)
        if weights is not None:
            self.load(weights)
        if weights is not None or checkpoint is not None:
            self.finalize()

    def load_safetensors(self, path):
        n = ctypes.c_int(0)
        _check(lib().ming_cuda_load_safetensors(self._h, os.fsencode(path), ctypes.byref(n)))
        return n.value

    def load(self, weights):
        for name, arr in weights.items():
            arr = np.ascontiguousarray(arr)
            shape = (ctypes.c_int64 * arr.ndim)(*arr.shape)
            _check(lib().ming_cuda_load_tensor(self._h, name.encode(), _dtype_code(arr), shape, arr.ndim, _ptr(arr)))

    def finalize(self):
        _check(lib().ming_cuda_finalize(self._h))

    def seq_alloc(self):
        s = ctypes.c_int()
        _check(lib().ming_cuda_seq_alloc(self._h, ctypes.byref(s)))
        return s.value

    def seq_free(self, s):
        _check(lib().ming_cuda_seq_free(self._h, s))

    def seq_len(self, s):
        n = ctypes.c_int()
        _check(lib().ming_cuda_seq_len(self._h, s, ctypes.byref(n)))
        return n.value

    def seq_truncate(self, s, n):
        _check(lib().ming_cuda_seq_truncate(self._h, s, n))

    def prefill(self, s, x, want_out=True):
        """x: uint16 [L, hidden] host array -> (out [L, hidden] uint16, stop [L] f32)."""
        x = np.ascontiguousarray(x, dtype=np.uint16)
        L = x.shape[0]
        out = np.empty_like(x) if want_out else None
        stop = np.empty(L, dtype=np.float32) if want_out else None
        _check(lib().ming_cuda_lm_prefill(self._h, s, _ptr(x), L, _ptr(out), _ptr(stop), PTR_HOST))
        return out, stop

    def decode(self, seqs, x):
        x = np.ascontiguousarray(x, dtype=np.uint16)
        B = len(seqs)
        ids = (ctypes.c_int * B)(*seqs)
        out = np.empty_like(x)
        stop = np.empty(B, dtype=np.float32)
        _check(lib().ming_cuda_lm_decode(self._h, B, ids, _ptr(x), _ptr(out), _ptr(stop), PTR_HOST))
        return out, stop

    def decode_noalloc(self, seqs, x):
        """One decode step without any device allocation (the attention
        scratch lives in a fixed array compiled into the library)."""
        x = np.ascontiguousarray(x, dtype=np.uint16)
        B = len(seqs)
        ids = (ctypes.c_int * B)(*seqs)
        out = np.empty_like(x)
        stop = np.empty(B, dtype=np.float32)
        _check(lib().ming_cuda_lm_decode_noalloc(self._h, B, ids, _ptr(x), _ptr(out), _ptr(stop), PTR_HOST))
        return out, stop

    def generate(self, seqs, x0, steps, kind=PTR_HOST, out=None, stop=None):
        """steps decode steps feeding each output back. Host mode returns
        (out [steps, B, hidden], stop [steps, B]); device mode takes device
        tensors (anything with data_ptr()) and returns them."""
        B = len(seqs)
        ids = (ctypes.c_int * B)(*seqs)
        if kind == PTR_HOST:
            x0 = np.ascontiguousarray(x0, dtype=np.uint16)
            if out is None:
                out = np.empty((steps, B, x0.shape[-1]), dtype=np.uint16)
            if stop is None:
                stop = np.empty((steps, B), dtype=np.float32)
        _check(lib().ming_cuda_lm_generate(self._h, B, ids, _ptr(x0), steps, _ptr(out), _ptr(stop), kind))
        return out, stop

    def cfm_sample(self, z, hist, noise, sde=None, cfg=2.0, shift=0.0):
        z = np.ascontiguousarray(z, dtype=np.uint16)
        B = z.shape[0]
        noise = np.ascontiguousarray(noise, dtype=np.uint16)
        y = np.empty_like(noise)
        _check(lib().ming_cuda_cfm_sample(self._h, B, _ptr(z), _ptr(None if hist is None else np.ascontiguousarray(hist)),
                                          _ptr(noise), _ptr(None if sde is None else np.ascontiguousarray(sde)),
                                          float(cfg), float(shift), _ptr(y), PTR_HOST))
        return y

    def cfm_steps(self, z, hist, y, step0, nsteps, sde=None, cfg=2.0, shift=0.0):
        z = np.ascontiguousarray(z, dtype=np.uint16)
        y = np.ascontiguousarray(y, dtype=np.uint16)
        out = np.empty_like(y)
        _check(lib().ming_cuda_cfm_steps(self._h, z.shape[0], _ptr(z), _ptr(None if hist is None else np.ascontiguousarray(hist)),
                                         _ptr(y), _ptr(None if sde is None else np.ascontiguousarray(sde)), float(cfg),
                                         float(shift), step0, nsteps, _ptr(out), PTR_HOST))
        return out

    def aggregate(self, latent):
        latent = np.ascontiguousarray(latent, dtype=np.uint16)
        B = latent.shape[0]
        out = np.empty((B, self.cfg.hidden), dtype=np.uint16)
        _check(lib().ming_cuda_aggregate(self._h, B, _ptr(latent), _ptr(out), PTR_HOST))
        return out

    def kv_read(self, s, layer, pos0, n):
        kh = self.cfg.kv_heads
        k = np.empty((kh, n, 64), dtype=np.uint16)
        v = np.empty((kh, n, 64), dtype=np.uint16)
        _check(lib().ming_cuda_kv_read(self._h, s, layer, pos0, n, _ptr(k), _ptr(v)))
        return k, v

    def _latent_width(self):
        return self.cfg.dit_frames * self.cfg.dit_latent

    def sample_latents(self, embeds, prompt_latent=None, params=None, bank=None, seed=0, trace=False):
        """sampleLatents: embeds [L, hidden] -> (latents [n, frames*latent],
        z trace [n, hidden] or None, stop trace [n]). bank: replay noise
        [steps, 11, frames*latent] or None (the library's seeded stream)."""
        embeds = np.ascontiguousarray(embeds, dtype=np.uint16)
        p = params if params is not None else sample_params()
        FL = self._latent_width()
        cap = p.max_steps
        bank_steps = 0
        if bank is not None:
            bank = np.ascontiguousarray(bank, dtype=np.uint16)
            bank_steps = bank.shape[0]
            cap = min(cap, bank_steps)
        lat = np.empty((cap, FL), dtype=np.uint16)
        zt = np.empty((cap, self.cfg.hidden), dtype=np.uint16) if trace else None
        st = np.empty(cap, dtype=np.float32)
        n = ctypes.c_int(0)
        pl = None if prompt_latent is None else np.ascontiguousarray(prompt_latent, dtype=np.uint16)
        _check(lib().ming_cuda_sample_latents(self._h, _ptr(embeds), embeds.shape[0], _ptr(pl), ctypes.byref(p), _ptr(bank),
                                              bank_steps, seed, _ptr(lat), cap, ctypes.byref(n), _ptr(zt), _ptr(st)))
        k = n.value
        return lat[:k], (zt[:k] if trace else None), st[:k]

    def vae_decode(self, latents):
        """Model.vaeDecode: latents uint16 bf16 [T, 64] -> waveform f32 [T * 4 * 882]."""
        latents = np.ascontiguousarray(latents, dtype=np.uint16)
        T = latents.shape[0]
        wave = np.empty(T * 4 * 882, dtype=np.float32)
        _check(lib().ming_cuda_vae_decode(self._h, _ptr(latents), T, _ptr(wave), PTR_HOST))
        return wave

    def kv_write(self, s, layer, pos0, k, v):
        """k, v: uint16 [kv_heads, n, 64] bf16 written at positions pos0.."""
        k = np.ascontiguousarray(k, dtype=np.uint16)
        v = np.ascontiguousarray(v, dtype=np.uint16)
        assert k.shape == v.shape and k.shape[0] == self.cfg.kv_heads and k.shape[2] == 64
        _check(lib().ming_cuda_kv_write(self._h, s, layer, pos0, k.shape[1], _ptr(k), _ptr(v)))

    def unpack_linear(self, weight_name, out_dim, in_dim):
        out = np.empty((out_dim, in_dim), dtype=np.float32)
        _check(lib().ming_cuda_unpack_linear(self._h, weight_name.encode(), _ptr(out)))
        return out

    def flow_temb(self):
        te = np.empty((10, self.cfg.dit_hidden), dtype=np.uint16)
        _check(lib().ming_cuda_flow_temb(self._h, _ptr(te)))
        return te

    @property
    def stream(self):
        s = ctypes.c_void_p()
        _check(lib().ming_cuda_get_stream(self._h, ctypes.byref(s)))
        return s.value

    def step_kernels(self, B):
        """Kernels one decode step of B rows launches (1 = persistent kernel)."""
        n = ctypes.c_int(0)
        _check(lib().ming_cuda_step_kernels(self._h, B, ctypes.byref(n)))
        return n.value

    def sync(self):
        _check(lib().ming_cuda_sync(self._h))

    def close(self):
        if self._h:
            lib().ming_cuda_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Loop:
    """ming_loop: the sampling loop over up to max_rows concurrent requests
    (continuous batching). submit() queues a request, step() runs one step
    of every active row, result() returns a finished request's latents."""

    def __init__(self, ctx, max_rows, params=None):
        self.ctx = ctx
        self.params = params if params is not None else sample_params()
        self._h = ctypes.c_void_p()
        _check(lib().ming_cuda_loop_create(ctx._h, max_rows, ctypes.byref(self.params), ctypes.byref(self._h)))

    def submit(self, embeds, prompt_latent=None, bank=None, seed=0, trace=False):
        embeds = np.ascontiguousarray(embeds, dtype=np.uint16)
        pl = None if prompt_latent is None else np.ascontiguousarray(prompt_latent, dtype=np.uint16)
        bank_steps = 0
        if bank is not None:
            bank = np.ascontiguousarray(bank, dtype=np.uint16)
            bank_steps = bank.shape[0]
        rid = ctypes.c_int(-1)
        _check(lib().ming_cuda_loop_submit(self._h, _ptr(embeds), embeds.shape[0], _ptr(pl), _ptr(bank), bank_steps, seed,
                                           1 if trace else 0, ctypes.byref(rid)))
        return rid.value

    def step(self):
        a, q = ctypes.c_int(0), ctypes.c_int(0)
        _check(lib().ming_cuda_loop_step(self._h, ctypes.byref(a), ctypes.byref(q)))
        return a.value, q.value

    def result(self, rid, trace=False):
        """None while the request runs; else (latents, z trace or None, stop trace)."""
        cap = self.params.max_steps
        FL = self.ctx._latent_width()
        lat = np.empty((cap, FL), dtype=np.uint16)
        zt = np.empty((cap, self.ctx.cfg.hidden), dtype=np.uint16) if trace else None
        st = np.empty(cap, dtype=np.float32)
        n = ctypes.c_int(0)
        _check(lib().ming_cuda_loop_result(self._h, rid, _ptr(lat), cap, ctypes.byref(n), _ptr(zt), _ptr(st)))
        if n.value < 0:
            return None
        k = n.value
        return lat[:k], (zt[:k] if trace else None), st[:k]

    def close(self):
        if self._h:
            lib().ming_cuda_loop_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
