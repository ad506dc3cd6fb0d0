"""The checkpoint reader (ming_cuda_load_safetensors, Model.load's file side,
src/ming_model.zig:316-350,923-1005).

CPU: files written by synth.save_safetensors validate without a context
(only the hot path's names and dtypes count), and malformed files are
rejected before any tensor is used. GPU: a context loaded from the file
decodes bit-identically to one loaded tensor by tensor; F32 / F16 copies of
bf16 tensors load as the same bf16 values; names off the hot path and
integer tables are skipped."""
import json
import os

import numpy as np
import pytest

import ming_b200 as M
from ming_b200 import synth


def _write_raw(path, header, blob=b""):
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        f.write(blob)


def test_validate_counts_hot_path_tensors(tmp_path):
    W = {
        "model.model.norm.weight": synth.ones_bf16((896,)),
        "stop_head.weight": synth.normal_bf16(1, "sw", (2, 896)),
        "flowloss.cfm.model.rotary_embed.inv_freq": synth.inv_freq(),
        "model.model.embed_tokens.index": np.arange(4, dtype=np.int32),  # integer table: skipped
        "audio.decoder.fc1.weight": synth.normal_bf16(1, "dec", (4, 4)),  # the VAE decoder: read
        "model.lm_head.weight": synth.normal_bf16(1, "lm_head", (4, 4)),  # not used by this library: skipped
    }
    p = tmp_path / "model.safetensors"
    synth.save_safetensors(p, W, metadata={"format": "mlx"})
    assert M.check_safetensors(str(p)) == 4
    assert M.check_safetensors(str(tmp_path)) == 4  # a model directory, as Model.load takes


@pytest.mark.parametrize("case", ["short", "hdr_len", "json", "offsets", "dtype", "shape", "trailing"])
def test_malformed_files_are_rejected(tmp_path, case):
    p = str(tmp_path / "bad.safetensors")
    good = {"stop_head.bias": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}}
    if case == "short":
        open(p, "wb").write(b"\x01\x02")
    elif case == "hdr_len":
        with open(p, "wb") as f:
            f.write((1 << 40).to_bytes(8, "little"))
            f.write(b"{}")
    elif case == "json":
        with open(p, "wb") as f:
            h = b'{"stop_head.bias": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]'
            f.write(len(h).to_bytes(8, "little"))
            f.write(h + b"\0\0\0\0")
    elif case == "offsets":
        _write_raw(p, {"stop_head.bias": {"dtype": "BF16", "shape": [3], "data_offsets": [0, 4]}}, b"\0" * 4)
    elif case == "dtype":
        _write_raw(p, {"stop_head.bias": {"dtype": "Q4", "shape": [2], "data_offsets": [0, 4]}}, b"\0" * 4)
    elif case == "shape":
        _write_raw(p, {"stop_head.bias": {"dtype": "BF16", "shape": [-2], "data_offsets": [0, 4]}}, b"\0" * 4)
    elif case == "trailing":
        _write_raw(p, good, b"\0" * 2)  # data shorter than the offsets say
    with pytest.raises(M.MingError):
        M.check_safetensors(p)


def test_missing_file_is_an_error(tmp_path):
    with pytest.raises(M.MingError, match="cannot open"):
        M.check_safetensors(str(tmp_path / "none.safetensors"))


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 16])
def test_checkpoint_loads_like_tensor_by_tensor(cuda_ok, tmp_path, bits):
    W = synth.lm_weights(seed=51, bits=bits, layers=2, qscale=(0.002, 0.005))
    F = dict(W)
    # float copies of bf16 tensors: the reader rounds them back to the same bf16
    F["model.model.norm.weight"] = synth.bf16_to_f32(W["model.model.norm.weight"])
    F["stop_head.bias"] = synth.bf16_to_f32(W["stop_head.bias"]).astype(np.float16)
    F["model.model.embed_tokens.weight"] = synth.normal_bf16(51, "emb", (16, 896))  # not read by the hot path
    F["audio.encoder.encoder.layers.0.mlp.down_proj.weight"] = synth.normal_bf16(51, "enc", (8, 8))
    p = str(tmp_path / "model.safetensors")
    synth.save_safetensors(p, F)
    cfg = M.default_cfg(layers=2, weight_bits=bits, dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=256, max_pages=64)
    a = M.Context(cfg, weights=W)
    b = M.Context(M.default_cfg(layers=2, weight_bits=bits, dit_mode=M.DIT_NONE, agg_blocks=0, max_ctx=256, max_pages=64),
                  checkpoint=str(tmp_path))
    x = synth.normal_bf16(52, "st.prompt", (9, 896))
    sa, sb = a.seq_alloc(), b.seq_alloc()
    oa, pa = a.prefill(sa, x)
    ob, pb = b.prefill(sb, x)
    assert np.array_equal(oa, ob) and np.array_equal(pa, pb)
    for _ in range(3):
        da, qa = a.decode([sa], oa[-1:])
        db, qb = b.decode([sb], ob[-1:])
        assert np.array_equal(da, db) and np.array_equal(qa, qb)
        oa, ob = da, db
    a.close()
    b.close()
