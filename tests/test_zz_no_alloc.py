"""fr_decode_attn_noalloc: decode attention that allocates no device memory.

Some callers of this library cannot call cudaMalloc: code that runs under
another framework's allocator or memory pool, plugins whose host process owns
every device allocation, or services that must not grow their device
footprint once started.  They use this entry point, whose split partial
states live in a static 1 MiB device array inside the library (and whose
in-kernel error word is a static device word too) instead of a workspace
grown with cudaMalloc.

Checked here, through the C ABI:
  * two calls in a row (different sizes, the second reusing the scratch the
    first left behind) agree with the regular entry point fr_decode_attn and
    with the CPU oracle at the engine's tolerance (max abs 2e-3, max rel 1e-2
    with a 1e-3 floor), and the static error word reads zero afterwards;
  * a problem whose partials exceed the static array is refused with
    FR_ERR_SCRATCH_LIMIT and launches nothing;
  * in a fresh process, further calls leave the device's free memory
    unchanged and the library's own cudaMalloc'd state empty.
This file is collected last, so a stop-at-first-failure run has already run
every other test.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from forgert_b200 import _lib
from forgert_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
ATOL, RTOL, EPS = 2e-3, 1e-2, 1e-3
SCRATCH_BYTES = 1 << 20          # FR_NOALLOC_SCRATCH_BYTES


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


def _planned_partial_bytes(H, Hkv, D, kv_len):
    """The allocation-free plan: one CTA per SM shared by the (kv head, head
    group) units, whole 64-row tiles per split."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    group = H // Hkv
    nt = 1 if group <= 8 else 2
    units = Hkv * -(-group // (8 * nt))
    tiles = -(-kv_len // 64)
    want = min(max(1, sms // units), tiles)
    tps = -(-tiles // want)
    splits = -(-tiles // tps)
    return H * splits * (D + 2) * 4 if splits > 1 else 0


def test_noalloc_matches_regular_entry_point_twice():
    lib = _lib.load()
    cases = [
        W.decode_inputs(101, 12, 2, 128, 16384),   # 64 splits: partials in the static array
        W.decode_inputs(102, 14, 2, 64, 3000),     # smaller, reuses what call 1 left behind
    ]
    for q, k, v in cases:
        st_na, out_na = _call(lib.fr_decode_attn_noalloc, q, k, v, k.shape[0])
        assert st_na == _lib.FR_OK, lib.fr_status_string(st_na)
        st_re, out_re = _call(lib.fr_decode_attn, q, k, v, k.shape[0])
        assert st_re == _lib.FR_OK
        _close(out_na, out_re, "noalloc vs fr_decode_attn")
        _close(out_na, O.decode_f64(q, k, v), "noalloc vs oracle")
    code = _lib.ctypes.c_int(-1)
    assert lib.fr_get_device_error(0, _lib.ctypes.byref(code)) == _lib.FR_OK
    assert code.value == 0


def test_noalloc_oversized_partials_refused():
    """16 query heads over one kv head at kv_len 16384: one CTA per SM gives
    128 splits on a 148-SM B200, 16 * 128 * 130 * 4 = 1.06 MB of partials,
    more than the 1 MiB array.  The call is refused before any launch: the
    NaN-filled output stays untouched."""
    H, Hkv, D, T = 16, 1, 128, 16384
    need = _planned_partial_bytes(H, Hkv, D, T)
    assert need > SCRATCH_BYTES, f"case must exceed the scratch on this device ({need} B)"
    lib = _lib.load()
    q, k, v = W.decode_inputs(103, H, Hkv, D, T)
    st, out = _call(lib.fr_decode_attn_noalloc, q, k, v, T)
    assert st == _lib.FR_ERR_SCRATCH_LIMIT, lib.fr_status_string(st)
    assert np.isnan(out.astype(np.float64)).all()
    assert b"scratch" in lib.fr_status_string(st)


_FRESH_PROCESS = r"""
import json, sys, ctypes
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
from forgert_b200 import _lib
from forgert_b200 import workloads as W
torch.cuda.set_device(0)
lib = _lib.load()
bufs = []
for seed, (H, Hkv, D, T) in enumerate([(12, 2, 128, 16384), (28, 4, 128, 8192), (14, 2, 64, 3000)]):
    q, k, v = W.decode_inputs(200 + seed, H, Hkv, D, T)
    qd, kd, vd = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, k, v))
    bufs.append((qd, kd, vd, torch.empty_like(qd), H, Hkv, D, T))
torch.cuda.synchronize()
def call(i):
    qd, kd, vd, out, H, Hkv, D, T = bufs[i]
    st = lib.fr_decode_attn_noalloc(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(),
                                     H, Hkv, D, T, None)
    torch.cuda.synchronize()
    return st
res = {"before_any": lib.fr_allocated_bytes(), "status": [call(0)]}
free0 = torch.cuda.mem_get_info()[0]
res["status"] += [call(1), call(2), call(0)]
code = ctypes.c_int(-1)
res["err_status"] = lib.fr_get_device_error(1, ctypes.byref(code))
res["err_code"] = code.value
free1 = torch.cuda.mem_get_info()[0]
res["free_delta"] = free0 - free1
res["after"] = lib.fr_allocated_bytes()
print(json.dumps(res))
"""


def test_noalloc_fresh_process_allocates_nothing():
    """In a process that never called the regular entry points, the library
    owns no cudaMalloc'd memory before or after allocation-free calls, and the
    calls after the first (whose one-time set-up looks up the static arrays)
    leave the device's free memory exactly unchanged."""
    r = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, str(ROOT)], capture_output=True,
                       text=True, timeout=600, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["status"] == [_lib.FR_OK] * 4, res
    assert res["err_status"] == _lib.FR_OK and res["err_code"] == 0, res
    assert res["before_any"] == 0 and res["after"] == 0, res
    assert res["free_delta"] == 0, res
