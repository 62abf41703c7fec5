"""RoPE tables against the reference's own table kernel, on one B200.

The reference builds its cos/sin tables on the GPU (kernels/rope.cu:28-56,
rope_precompute_tables) with --use_fast_math, i.e. with the fast approximate
sine and cosine, whose error grows with the angle theta = pos / base^(2f/D)
(up to ~16383 rad at position 16383).  Checked here, on the reference's
kernel compiled from its sources (oracle/_ref):

* fr_rope_tables_device reproduces the reference tables bit for bit at
  max_seq_len 16384, theta_base 1e6, head_dim 128 and 64;
* fr_rope_tables (exactly rounded, fp64 on the host) differs from them by
  the fast functions' error; the rotated q/k of the reference's own
  rope_v2_fused with the two table sets are compared in fp16 ulps, and the
  figures are printed (pytest -s): the exact tables are the more accurate,
  the device tables the ones that match the reference engine.
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

S = 16384


@pytest.fixture(scope="module")
def ref():
    lib = O.load_ref()
    if lib is None:
        pytest.skip("oracle/_ref not built")
    return lib


def ref_tables(ref, D, theta=W.ROPE_THETA):
    c = torch.empty((S, D // 2), dtype=torch.float32, device="cuda")
    s = torch.empty_like(c)
    assert ref.ref_rope_precompute_tables(c.data_ptr(), s.data_ptr(), S, D, theta, 1.0) == 0
    torch.cuda.synchronize()
    return c, s


@pytest.mark.parametrize("D", [128, 64])
def test_device_tables_match_reference_bit_for_bit(ref, D):
    rc, rs = ref_tables(ref, D)
    oc, os_ = A.rope_tables_device(S, D, W.ROPE_THETA)
    torch.cuda.synchronize()
    bad_c = int((oc.view(torch.int32) != rc.view(torch.int32)).sum())
    bad_s = int((os_.view(torch.int32) != rs.view(torch.int32)).sum())
    assert bad_c == 0 and bad_s == 0, (bad_c, bad_s, float((oc - rc).abs().max()),
                                       float((os_ - rs).abs().max()))


def _ulps(a: torch.Tensor, b: torch.Tensor) -> np.ndarray:
    """|a - b| in fp16 ulps of b (ordered-integer distance of the bit patterns)."""
    def ordered(x):
        i = x.view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -32768 - i, i)
    return (ordered(a) - ordered(b)).abs().cpu().numpy()


@pytest.mark.parametrize("H,Hkv,D", [(12, 2, 128), (14, 2, 64)])
def test_exact_tables_vs_reference_tables(ref, H, Hkv, D):
    rc, rs = ref_tables(ref, D)
    ec, es = A.rope_precompute_tables(S, D, W.ROPE_THETA)
    torch.cuda.synchronize()
    dcos = (ec - rc).abs()
    dsin = (es - rs).abs()
    # rotate the same q/k at every position 0..S-1 with the reference kernel
    rng = np.random.default_rng(21)
    q0 = torch.from_numpy(W.normal_fp16(rng, (S, H, D))).cuda()
    k0 = torch.from_numpy(W.normal_fp16(rng, (S, Hkv, D))).cuda()
    outs = []
    for c, s in ((rc, rs), (ec, es)):
        q, k = q0.clone(), k0.clone()
        ref.ref_rope_v2_fused(q.data_ptr(), k.data_ptr(), c.data_ptr(), s.data_ptr(), S, H, Hkv,
                              D, 0, None)
        outs.append((q, k))
    torch.cuda.synchronize()
    uq = _ulps(outs[1][0], outs[0][0])
    uk = _ulps(outs[1][1], outs[0][1])
    by_pos = uq.reshape(S, -1).max(axis=1)
    stats = {
        "shape": f"H{H} Hkv{Hkv} D{D}, positions 0..{S - 1}, theta 1e6",
        "max_abs_dcos": float(dcos.max()), "max_abs_dsin": float(dsin.max()),
        "max_abs_dcos_pos_lt_512": float(dcos[:512].max()),
        "q_max_abs_diff": float((outs[1][0].float() - outs[0][0].float()).abs().max()),
        "q_max_ulp": int(uq.max()), "k_max_ulp": int(uk.max()),
        "q_frac_differing": round(float((uq > 0).mean()), 6),
        "q_frac_over_1ulp": round(float((uq > 1).mean()), 6),
        "first_pos_over_1ulp": int(np.argmax(by_pos > 1)) if (by_pos > 1).any() else None,
    }
    print("\n" + json.dumps({"rope_tables_exact_vs_reference": stats}))
    # the fast functions' error is bounded: the tables agree to a few 1e-3
    # (about 7e-5 already below position 512), and so do the rotated values
    assert stats["max_abs_dcos"] < 1e-2 and stats["max_abs_dsin"] < 1e-2
    assert stats["max_abs_dcos_pos_lt_512"] < 1e-3
    assert stats["q_max_abs_diff"] < 0.1
