"""CPU tests of the C ABI: the library loads, exports every function
include/ming_cuda.h declares, and rejects bad configurations before touching
a GPU."""
import ctypes
import os
import re

import pytest

import ming_b200 as M

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ensure_built():
    if not os.path.exists(M.LIB_PATH):
        import importlib.util
        spec = importlib.util.spec_from_file_location("ming_build", os.path.join(ROOT, "ming-tts-serve_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()


def header_functions():
    txt = open(os.path.join(ROOT, "include", "ming_cuda.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ming_cuda_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    _ensure_built()
    lib = ctypes.CDLL(M.LIB_PATH)
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding covers the same set
    assert sorted(M.SYMBOLS) == names


def test_default_cfg_is_the_reference_shape():
    _ensure_built()
    c = M.default_cfg()
    # Qwen2-0.5B LM of Ming-3.0-tts (src/ming_model.zig:37-53,500-504)
    assert (c.hidden, c.layers, c.heads, c.kv_heads, c.head_dim, c.ff) == (896, 24, 14, 2, 64, 4864)
    assert abs(c.rope_theta - 1e6) < 1 and abs(c.rms_eps - 1e-6) < 1e-9
    assert c.page_size == 16 and c.group_size == 64
    # reference flow head: 8 blocks x 1024, 16 heads, MLP 4096, latent 64
    assert (c.dit_mode, c.dit_hidden, c.dit_blocks, c.dit_heads, c.dit_ff, c.dit_latent) == (M.DIT_TOKEN, 1024, 8, 16, 4096, 64)


@pytest.mark.parametrize("field,value", [("head_dim", 32), ("page_size", 8), ("group_size", 32), ("kv_heads", 3),
                                         ("max_ctx", 1000), ("max_batch", 0)])
def test_create_rejects_bad_config(field, value):
    _ensure_built()
    c = M.default_cfg(**{field: value})
    h = ctypes.c_void_p()
    rc = M.lib().ming_cuda_create(0, ctypes.byref(c), ctypes.byref(h))
    assert rc == 1  # MING_ERR_INVALID, before any CUDA call
    assert M.lib().ming_cuda_last_error()


def test_null_arguments_are_errors():
    _ensure_built()
    L = M.lib()
    assert L.ming_cuda_create(0, None, None) == 1
    assert L.ming_cuda_finalize(None) == 1
    assert L.ming_cuda_sync(None) == 1
    assert L.ming_cuda_destroy(None) == 0


def test_every_call_rejects_a_null_context():
    """Each entry point checks its context before any CUDA call and returns
    MING_ERR_INVALID with a message, as the reference's check(rc) expects."""
    _ensure_built()
    L = M.lib()
    i32, u16, f32 = ctypes.c_int(0), (ctypes.c_uint16 * 8)(), (ctypes.c_float * 8)()
    ids = (ctypes.c_int * 1)(0)
    calls = {
        "seq_alloc": lambda: L.ming_cuda_seq_alloc(None, ctypes.byref(i32)),
        "seq_free": lambda: L.ming_cuda_seq_free(None, 0),
        "seq_len": lambda: L.ming_cuda_seq_len(None, 0, ctypes.byref(i32)),
        "seq_truncate": lambda: L.ming_cuda_seq_truncate(None, 0, 0),
        "lm_prefill": lambda: L.ming_cuda_lm_prefill(None, 0, u16, 1, u16, f32, 0),
        "lm_decode": lambda: L.ming_cuda_lm_decode(None, 1, ids, u16, u16, f32, 0),
        "lm_decode_noalloc": lambda: L.ming_cuda_lm_decode_noalloc(None, 1, ids, u16, u16, f32, 0),
        "lm_generate": lambda: L.ming_cuda_lm_generate(None, 1, ids, u16, 1, u16, f32, 0),
        "cfm_sample": lambda: L.ming_cuda_cfm_sample(None, 1, u16, u16, u16, None, ctypes.c_float(2.0), ctypes.c_float(0.0),
                                                     u16, 0),
        "cfm_steps": lambda: L.ming_cuda_cfm_steps(None, 1, u16, u16, u16, None, ctypes.c_float(2.0), ctypes.c_float(0.0),
                                                   0, 1, u16, 0),
        "aggregate": lambda: L.ming_cuda_aggregate(None, 1, u16, u16, 0),
        "kv_read": lambda: L.ming_cuda_kv_read(None, 0, 0, 0, 1, u16, u16),
        "step_kernels": lambda: L.ming_cuda_step_kernels(None, 1, ctypes.byref(i32)),
        "flow_temb": lambda: L.ming_cuda_flow_temb(None, u16),
    }
    for name, call in calls.items():
        assert call() == 1, name
        assert L.ming_cuda_last_error(), name
