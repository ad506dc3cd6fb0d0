"""Generates the golden fixtures that pin the CPU oracle.

The reference (Zig + MLX + Metal) cannot run in this container, so the LM's
algorithm is pinned against Hugging Face transformers' Qwen2 — the model the
reference's MLX graph mirrors op for op (src/ming_model.zig:566-614; "mirrors
the Python engine op for op", README.md:225) — run in fp32 on the same seeded
weights the oracle and the CUDA path use. The oracle's F32 mode (no bf16
rounding) must match these hidden states to fp32 rounding.

Fixture: lm_hf_f32.npz
  seed, layers, prefill, decode   workload description (weights/inputs are
                                   regenerated from ming_b200.synth)
  hidden [prefill+decode, 896]     post-final-norm hidden of every position
                                   (prefill rows, then each decode step fed
                                   the fixed decode inputs)

Run from the repo root: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "ming-tts-serve_b200"))
from ming_b200 import synth  # noqa: E402

SEED, LAYERS, PREFILL, DECODE = 0, 2, 6, 3


def lm_inputs(seed=SEED, n=PREFILL + DECODE, hidden=896):
    return synth.normal_bf16(seed, "golden.lm.inputs", (n, hidden), 1.0)


def main():
    import torch
    from transformers import Qwen2Config, Qwen2Model

    W = synth.lm_weights(seed=SEED, bits=16, layers=LAYERS)
    cfg = Qwen2Config(hidden_size=896, intermediate_size=4864, num_hidden_layers=LAYERS, num_attention_heads=14,
                      num_key_value_heads=2, head_dim=64, rope_theta=1e6, rms_norm_eps=1e-6, vocab_size=16,
                      max_position_embeddings=4096, attn_implementation="eager")
    model = Qwen2Model(cfg).eval().to(torch.float32)
    sd = {}
    f = lambda a: torch.from_numpy(synth.bf16_to_f32(a).copy())
    for l in range(LAYERS):
        p = f"model.model.layers.{l}"
        q = f"layers.{l}"
        sd[q + ".input_layernorm.weight"] = f(W[p + ".input_layernorm.weight"])
        sd[q + ".post_attention_layernorm.weight"] = f(W[p + ".post_attention_layernorm.weight"])
        for n in ("q_proj", "k_proj", "v_proj"):
            sd[f"{q}.self_attn.{n}.weight"] = f(W[f"{p}.self_attn.{n}.weight"])
            sd[f"{q}.self_attn.{n}.bias"] = f(W[f"{p}.self_attn.{n}.bias"])
        sd[q + ".self_attn.o_proj.weight"] = f(W[p + ".self_attn.o_proj.weight"])
        for n in ("gate_proj", "up_proj", "down_proj"):
            sd[f"{q}.mlp.{n}.weight"] = f(W[f"{p}.mlp.{n}.weight"])
    sd["norm.weight"] = f(W["model.model.norm.weight"])
    sd["embed_tokens.weight"] = torch.zeros(16, 896)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in m for m in missing), missing
    x = torch.from_numpy(synth.bf16_to_f32(lm_inputs()).copy()).reshape(1, PREFILL + DECODE, 896)
    from transformers import DynamicCache
    cache = DynamicCache()
    outs = []
    with torch.no_grad():
        o = model(inputs_embeds=x[:, :PREFILL], past_key_values=cache, use_cache=True)
        outs.append(o.last_hidden_state[0])
        for i in range(DECODE):
            o = model(inputs_embeds=x[:, PREFILL + i:PREFILL + i + 1], past_key_values=cache, use_cache=True)
            outs.append(o.last_hidden_state[0])
    hidden = torch.cat(outs, 0).numpy().astype(np.float32)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lm_hf_f32.npz")
    np.savez_compressed(out, seed=SEED, layers=LAYERS, prefill=PREFILL, decode=DECODE, hidden=hidden,
                        generator=np.array(f"transformers {__import__('transformers').__version__}, torch {torch.__version__}"))
    print("wrote", out, hidden.shape)


if __name__ == "__main__":
    main()
