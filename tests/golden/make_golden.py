"""Generates the golden vectors in tests/golden/ from the reference itself.

Run where the reference tree is available (it needs oracle/_ref, built by
`make -C oracle REF=<reference tree>`, and the `transformers` package):

    python tests/golden/make_golden.py

Each decode fixture stores the fp16 inputs and three outputs:
  ref_f32   the reference's own CPU oracle cpu_decode_attn
            (tests/test_kernels.cpp:229-270), compiled from its sources;
  hf_f16    transformers' Qwen2 eager_attention_forward on CPU in fp16 -
            the arithmetic of the reference's python/reference.py;
  exact     numpy fp64 of the same inputs (oracle/oracle.py decode_f64).
The prefill fixture stores hf_f16 (eager attention with a causal mask) and
exact; the RoPE fixture stores transformers' apply_rotary_pos_emb output.
Inputs that are cheap to regenerate (cfg1) are stored together with a
SHA-256 of their bytes, so a drift of the numpy generator is detected.
"""
from __future__ import annotations

import hashlib
import sys
import types
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from forgert_b200 import workloads as W  # noqa: E402
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def hf_decode(q, k, v):
    import torch
    from transformers.models.qwen2.modeling_qwen2 import eager_attention_forward

    H, D = q.shape
    Hkv = k.shape[1]
    mod = types.SimpleNamespace(num_key_value_groups=H // Hkv, training=False)
    qt = torch.from_numpy(q.copy()).view(1, H, 1, D)
    kt = torch.from_numpy(np.ascontiguousarray(k.transpose(1, 0, 2))).unsqueeze(0)
    vt = torch.from_numpy(np.ascontiguousarray(v.transpose(1, 0, 2))).unsqueeze(0)
    out, _ = eager_attention_forward(mod, qt, kt, vt, None, scaling=D ** -0.5)
    return out.reshape(H, D).numpy()


def hf_prefill(q, k, v):
    import torch
    from transformers.models.qwen2.modeling_qwen2 import eager_attention_forward

    T, H, D = q.shape
    Hkv = k.shape[1]
    mod = types.SimpleNamespace(num_key_value_groups=H // Hkv, training=False)
    qt = torch.from_numpy(np.ascontiguousarray(q.transpose(1, 0, 2))).unsqueeze(0)
    kt = torch.from_numpy(np.ascontiguousarray(k.transpose(1, 0, 2))).unsqueeze(0)
    vt = torch.from_numpy(np.ascontiguousarray(v.transpose(1, 0, 2))).unsqueeze(0)
    mask = torch.triu(torch.full((T, T), float("-inf")), 1).to(torch.float16)[None, None]
    out, _ = eager_attention_forward(mod, qt, kt, vt, mask, scaling=D ** -0.5)
    return out.reshape(T, H, D).numpy()


def hf_rope(x, pos, head_dim, theta):
    import torch
    from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = torch.tensor(pos, dtype=torch.float32)[:, None] * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos().to(torch.float16), emb.sin().to(torch.float16)
    xt = torch.from_numpy(x.copy())  # [T, heads, D]
    out, _ = apply_rotary_pos_emb(xt, xt, cos, sin, unsqueeze_dim=1)
    return out.numpy()


def decode_fixture(name, q, k, v, store_inputs=True, extra=None):
    ref = O.ref_cpu_decode_attn(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32))
    hf = hf_decode(q, k, v)
    exact = O.decode_f64(q, k, v)
    H, D = q.shape
    meta = dict(H=H, Hkv=k.shape[1], D=D, kv_len=k.shape[0], inputs_sha256=sha(q, k, v))
    arrays = dict(ref_f32=ref, hf_f16=hf, exact=exact)
    if store_inputs:
        arrays.update(q=q, k=k, v=v)
    if extra:
        meta.update(extra)
    np.savez_compressed(OUT / f"{name}.npz", meta=np.array(repr(meta)), **arrays)
    print(f"{name}: ref-vs-exact {O.max_errors(ref, exact)}, hf-vs-exact {O.max_errors(hf, exact)}")


def main() -> None:
    if O.load_ref() is None:
        sys.exit("oracle/_ref/libforgert_ref.so is missing: make -C oracle REF=<reference tree>")
    # The reference's own test shapes (tests/test_kernels.cpp:298-339), U(-0.5, 0.5).
    q, k, v = W.decode_inputs(12345, 8, 2, 64, 128, dist="uniform")
    decode_fixture("ref_h8_kv2_d64_len128", q, k, v)
    q1, k1, v1 = W.decode_inputs(12346, 8, 2, 64, 1, dist="uniform")
    decode_fixture("ref_h8_kv2_d64_len1", q1, k1, v1)
    q2, k2, v2 = W.decode_inputs(12347, 8, 2, 128, 128, dist="uniform")
    decode_fixture("ref_h8_kv2_d128_len128", q2, k2, v2)
    # BASELINE config 1 (inputs regenerated from seed 0; checksum stored).
    q, k, v = W.cfg1_inputs()
    decode_fixture("cfg1_h14_kv2_d64_len512", q, k, v, store_inputs=False,
                   extra=dict(generator="forgert_b200.workloads.cfg1_inputs"))
    # Shapes that exercise the kernel's edges: group 7 with a ragged tail,
    # group 16 (two 8-head tiles), MHA (group 1), group 6 (config 2 shape).
    for name, seed, H, Hkv, D, T in [
        ("gqa7_d128_len33", 21, 28, 4, 128, 33),
        ("gqa16_d64_len200", 22, 32, 2, 64, 200),
        ("mha_d128_len100", 23, 4, 4, 128, 100),
        ("gqa6_d128_len300", 24, 12, 2, 128, 300),
    ]:
        q, k, v = W.decode_inputs(seed, H, Hkv, D, T)
        decode_fixture(name, q, k, v)
    # Prefill (causal), cfg1 head shape.
    rng = np.random.default_rng(31)
    T, H, Hkv, D = 37, 14, 2, 64
    qp = W.normal_fp16(rng, (T, H, D))
    kp = W.normal_fp16(rng, (T, Hkv, D))
    vp = W.normal_fp16(rng, (T, Hkv, D))
    np.savez_compressed(OUT / "prefill_t37_h14_kv2_d64.npz", q=qp, k=kp, v=vp,
                        hf_f16=hf_prefill(qp, kp, vp), exact=O.prefill_f64(qp, kp, vp))
    # RoPE: tokens at positions 40..43, D 64, theta 1e6 (cfg5 shape).
    rng = np.random.default_rng(32)
    xr = W.normal_fp16(rng, (4, 14, 64))
    pos = [40, 41, 42, 43]
    np.savez_compressed(OUT / "rope_d64_pos40.npz", x=xr, pos=np.array(pos),
                        hf_f16=hf_rope(xr, pos, 64, W.ROPE_THETA), theta=W.ROPE_THETA)
    print("fixtures written to", OUT)


if __name__ == "__main__":
    main()
