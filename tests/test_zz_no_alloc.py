"""fr_decode_attn_noalloc: decode attention that allocates no device memory.

Callers that cannot call cudaMalloc (code running under another framework's
allocator or memory pool, plugins whose host owns every device allocation)
use this entry point; its split partial states live in a static 2 MiB device
array inside the library instead of a workspace grown with cudaMalloc.

The test calls it through the C ABI twice in a row (different sizes, the
second call reusing the scratch the first one left behind) and checks each
output against the regular entry point fr_decode_attn and against the CPU
oracle, at the engine's tolerance (max abs 2e-3, max rel 1e-2 with a 1e-3
floor).  A problem whose partials would exceed the static array is refused
with FR_ERR_SCRATCH_LIMIT before anything is launched.  This file is collected last so
a stop-at-first-failure run has already run every other test.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from forgert_b200 import _lib
from forgert_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL, EPS = 2e-3, 1e-2, 1e-3


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _call(fn, q, k, v, kv_len):
    H, D = q.shape
    Hkv = k.shape[1]
    qd, kd, vd = _dev(q), _dev(k), _dev(v)
    out = torch.full_like(qd, float("nan"))
    status = fn(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(), H, Hkv, D, kv_len,
                None)
    torch.cuda.synchronize()
    return status, out.cpu().numpy()


def _close(x, ref, what):
    a, r = O.max_errors(x, ref, EPS)
    assert np.isfinite(x.astype(np.float64)).all(), what
    assert a <= ATOL and r <= RTOL, f"{what}: max abs {a:.3g}, max rel {r:.3g}"


def test_noalloc_matches_regular_entry_point_twice():
    lib = _lib.load()
    cases = [
        W.decode_inputs(101, 12, 2, 128, 16384),   # 128 splits: partials in the static array
        W.decode_inputs(102, 14, 2, 64, 3000),     # smaller, reuses what call 1 left behind
    ]
    for q, k, v in cases:
        st_na, out_na = _call(lib.fr_decode_attn_noalloc, q, k, v, k.shape[0])
        assert st_na == _lib.FR_OK, lib.fr_status_string(st_na)
        st_re, out_re = _call(lib.fr_decode_attn, q, k, v, k.shape[0])
        assert st_re == _lib.FR_OK
        _close(out_na, out_re, "noalloc vs fr_decode_attn")
        _close(out_na, O.decode_f64(q, k, v), "noalloc vs oracle")


def test_noalloc_oversized_partials_refused_cleanly():
    """32 heads over 2 kv heads at kv_len 16384 plans ~2.1 MB of partials with
    two CTAs per SM (more than the 2 MiB array); the split count follows the
    device's occupancy, so either outcome is accepted, each checked: a
    refusal launches nothing, an accepted call is correct."""
    lib = _lib.load()
    q, k, v = W.decode_inputs(103, 32, 2, 128, 16384)
    st, out = _call(lib.fr_decode_attn_noalloc, q, k, v, k.shape[0])
    if st == _lib.FR_ERR_SCRATCH_LIMIT:
        assert np.isnan(out.astype(np.float64)).all()      # nothing was launched
        assert b"scratch" in lib.fr_status_string(st)
    else:
        assert st == _lib.FR_OK, lib.fr_status_string(st)
        _close(out, O.decode_f64(q, k, v), "noalloc (fits on this device)")
