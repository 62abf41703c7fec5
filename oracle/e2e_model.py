"""Random-init Qwen2-0.5B checkpoint for the end-to-end parity harness.

TEST INFRASTRUCTURE ONLY.  Writes <dir>/model.safetensors in the format the
reference loader reads (runtime/model.cpp:35-60, 132-254): HF tensor names,
F16 data, tied embeddings (no lm_head.weight, model.cpp:184, 221-225).
Weights are N(0, 0.02) fp16 drawn from numpy default_rng(4) in the order the
tensors are listed below; q/k/v biases are zero and RMSNorm weights one (the
HF initialisation), so both engines read identical bytes.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

VOCAB, HIDDEN, HEADS, KV_HEADS, HEAD_DIM, LAYERS, INTER = 151936, 896, 14, 2, 64, 24, 4864
PROMPT_LEN = 5


def tensor_list():
    kvd = KV_HEADS * HEAD_DIM
    out = [("model.embed_tokens.weight", (VOCAB, HIDDEN), "normal"),
           ("model.norm.weight", (HIDDEN,), "ones")]
    for l in range(LAYERS):
        p = f"model.layers.{l}"
        out += [
            (f"{p}.input_layernorm.weight", (HIDDEN,), "ones"),
            (f"{p}.post_attention_layernorm.weight", (HIDDEN,), "ones"),
            (f"{p}.self_attn.q_proj.weight", (HIDDEN, HIDDEN), "normal"),
            (f"{p}.self_attn.k_proj.weight", (kvd, HIDDEN), "normal"),
            (f"{p}.self_attn.v_proj.weight", (kvd, HIDDEN), "normal"),
            (f"{p}.self_attn.o_proj.weight", (HIDDEN, HIDDEN), "normal"),
            (f"{p}.self_attn.q_proj.bias", (HIDDEN,), "zeros"),
            (f"{p}.self_attn.k_proj.bias", (kvd,), "zeros"),
            (f"{p}.self_attn.v_proj.bias", (kvd,), "zeros"),
            (f"{p}.mlp.gate_proj.weight", (INTER, HIDDEN), "normal"),
            (f"{p}.mlp.up_proj.weight", (INTER, HIDDEN), "normal"),
            (f"{p}.mlp.down_proj.weight", (HIDDEN, INTER), "normal"),
        ]
    return out


def write_model(dirpath, seed: int = 4, std: float = 0.02) -> Path:
    d = Path(dirpath)
    d.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    header, off = {}, 0
    specs = tensor_list()
    for name, shape, _ in specs:
        n = int(np.prod(shape)) * 2
        header[name] = {"dtype": "F16", "shape": list(shape), "data_offsets": [off, off + n]}
        off += n
    hbytes = json.dumps(header).encode()
    hbytes += b" " * ((8 - len(hbytes) % 8) % 8)
    path = d / "model.safetensors"
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hbytes)))
        f.write(hbytes)
        for name, shape, kind in specs:
            if kind == "normal":
                a = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float16)
            elif kind == "ones":
                a = np.ones(shape, np.float16)
            else:
                a = np.zeros(shape, np.float16)
            f.write(a.tobytes())
    return path


def prompt_ids(seed: int = 4) -> list[int]:
    return [int(x) for x in np.random.default_rng([seed, 1]).integers(0, VOCAB, PROMPT_LEN)]
