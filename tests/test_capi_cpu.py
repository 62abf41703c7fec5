"""The C-ABI boundary, checked without a GPU.

* libforgert_b200.so loads and exports every function include/forgert_attn.h
  declares (and the ctypes table covers exactly that set);
* argument validation answers with the documented status codes before any
  CUDA call (so these run on a CPU-only machine);
* include/forgert_attn.h is plain C, and include/attention.cuh - the C++
  drop-in for the reference's kernels/attention.cuh - compiles the
  reference's runtime/executor.cpp unchanged and links against the library.
"""
from __future__ import annotations

import ctypes
import os
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from forgert_b200 import _lib
from forgert_b200 import attention as A
from oracle import paths

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "forgert_attn.h"
REF = paths.reference_tree() or Path("/nonexistent")
# the CUDA toolkit's headers, next to the nvcc on PATH
CUDA_INC = str(Path(shutil.which("nvcc") or "nvcc").resolve().parent.parent / "include")


def header_symbols():
    text = HEADER.read_text()
    return set(re.findall(r"FR_API\s+[\w\s\*]+?\b(fr_\w+)\s*\(", text))


def test_every_declared_symbol_is_exported(lib):
    names = header_symbols()
    assert len(names) >= 14
    nm = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                        text=True, check=True).stdout
    exported = set(re.findall(r"\bT (fr_\w+)", nm))
    assert names <= exported, names - exported
    assert exported <= names, f"exported but undeclared: {exported - names}"
    assert set(_lib.SIGNATURES) == names
    for n in names:
        assert getattr(lib, n) is not None


def test_version_and_status_strings(lib):
    assert lib.fr_version() == 100
    for st in range(0, 8):
        assert lib.fr_status_string(st)
    assert lib.fr_launch_count() >= 0


def test_validation_before_any_cuda_call(lib):
    nullp = None
    fake = 0x10000       # never dereferenced: validation rejects first
    # null pointers / bad sizes -> FR_ERR_INVALID_ARG
    assert lib.fr_decode_attn(nullp, fake, fake, fake, 8, 2, 64, 16, None) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_decode_attn(fake, fake, fake, fake, 8, 2, 64, 0, None) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_decode_attn(fake, fake, fake, fake, 8, 3, 64, 16, None) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_decode_attn(fake, fake, fake, fake, 0, 1, 64, 16, None) == _lib.FR_ERR_INVALID_ARG
    # head_dim outside {64, 128} -> FR_ERR_UNSUPPORTED (the reference silently fell back to v3)
    assert lib.fr_decode_attn(fake, fake, fake, fake, 8, 2, 96, 16, None) == _lib.FR_ERR_UNSUPPORTED
    assert lib.fr_decode_attn(fake, fake, fake, fake, 8, 2, 256, 16, None) == _lib.FR_ERR_UNSUPPORTED
    # TMA bulk copies need 16-byte aligned k/v
    assert lib.fr_decode_attn(fake, fake + 8, fake, fake, 8, 2, 64, 16, None) == _lib.FR_ERR_MISALIGNED
    assert lib.fr_decode_attn(fake + 2, fake, fake, fake, 8, 2, 64, 16, None) == _lib.FR_ERR_MISALIGNED
    assert lib.fr_prefill_attn(fake, fake, fake, fake, 0, 8, 2, 64, None) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_decode_attn_batched(fake, fake, fake, fake, fake, fake, 0, 8, 2, 64, 100, 16,
                                      None) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_decode_attn_batched(fake, fake + 8, fake, fake, fake, fake, 2, 8, 2, 64, 100, 16,
                                      None) == _lib.FR_ERR_MISALIGNED
    # paged: page_size a multiple of 16, the table must cover max_kv_len, pool < 2^31 rows
    paged = lambda *a: lib.fr_decode_attn_paged(fake, fake, fake, fake, fake, fake, *a, None)  # noqa: E731
    assert paged(2, 8, 2, 64, 8, 10, 4, 32) == _lib.FR_ERR_INVALID_ARG
    assert paged(2, 8, 2, 64, 24, 10, 4, 64) == _lib.FR_ERR_INVALID_ARG
    assert paged(2, 8, 2, 64, 16, 10, 4, 65) == _lib.FR_ERR_INVALID_ARG
    assert paged(2, 8, 2, 64, 16, 0, 4, 64) == _lib.FR_ERR_INVALID_ARG
    assert paged(0, 8, 2, 64, 16, 10, 4, 64) == _lib.FR_ERR_INVALID_ARG
    assert paged(2, 8, 2, 64, 1 << 16, 1 << 15, 4, 64) == _lib.FR_ERR_INVALID_ARG
    assert paged(2, 8, 2, 96, 16, 10, 4, 64) == _lib.FR_ERR_UNSUPPORTED
    assert lib.fr_decode_attn_paged(fake, fake + 8, fake, fake, fake, fake, 2, 8, 2, 64, 16, 10,
                                    4, 64, None) == _lib.FR_ERR_MISALIGNED
    assert lib.fr_decode_attn_partial(fake, fake, fake, -1, fake, fake, 8, 2, 64, None) == \
        _lib.FR_ERR_INVALID_ARG
    assert lib.fr_lse_merge(fake, fake, 0, fake, 8, 64, None) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_lse_merge_strided(fake, fake, 2, fake, 8, 64, 3, 64, None) == _lib.FR_ERR_MISALIGNED
    assert lib.fr_rope_tables(None, None, 16, 64, 1e6, 1.0) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_rope_append(fake, fake, fake, fake, fake, fake, fake, 1, 8, 2, 64, -1, None) == \
        _lib.FR_ERR_INVALID_ARG
    # prefill: q/k/v are TMA-copied (16-byte aligned), head_dim in {64, 128}
    assert lib.fr_prefill_attn(fake + 4, fake, fake, fake, 16, 8, 2, 64, None) == _lib.FR_ERR_MISALIGNED
    assert lib.fr_prefill_attn(fake, fake, fake, fake, 16, 8, 2, 96, None) == _lib.FR_ERR_UNSUPPORTED
    assert lib.fr_prefill_workspace_size(0, 8, 64) == 0
    assert lib.fr_prefill_workspace_size(16, 8, 96) == 0
    # kernel copy: zero bytes is a no-op, null pointers are refused
    assert lib.fr_copy_async(fake, fake, 0, None) == _lib.FR_OK
    assert lib.fr_copy_async(nullp, fake, 16, None) == _lib.FR_ERR_INVALID_ARG
    assert lib.fr_copy_async(fake, nullp, 16, None) == _lib.FR_ERR_INVALID_ARG


def test_python_mirror_raises_like_cuda_check():
    with pytest.raises(_lib.ForgeRTError) as e:
        A.decode_attn_v4_flash(0x10000, 0x10008, 0x10000, 0x10000, 8, 2, 64, 16)
    assert e.value.status == _lib.FR_ERR_MISALIGNED
    assert isinstance(e.value, RuntimeError)
    # the reference's older versions are the same entry point
    assert A.decode_attn_v3_vec is A.decode_attn_v4_flash
    # copy_async reaches host memory only through a page-locked mapping
    import torch
    with pytest.raises(ValueError):
        A.copy_async(torch.zeros(4), torch.zeros(4))


def test_c_header_is_plain_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "forgert_attn.h"\nint main(void){return fr_version() > 0 ? 0 : 1;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-I",
                    str(ROOT / "include"), str(src)], check=True)


@pytest.mark.skipif(not shutil.which("g++"), reason="g++ missing")
def test_shim_links_against_library(tmp_path):
    """A C++ caller of the drop-in header links against libforgert_b200.so."""
    src = tmp_path / "caller.cpp"
    src.write_text(
        '#include "attention.cuh"\n'
        "void f(const __half* q, const __half* k, const __half* v, __half* o) {\n"
        "  decode_attn_v4_flash(q, k, v, o, 14, 2, 64, 512);\n"
        "  decode_attn_v0_naive(q, k, v, o, 14, 2, 64, 512, nullptr);\n"
        "  prefill_attn_causal(q, k, v, o, 5, 14, 2, 64);\n"
        "}\nint main() { return 0; }\n")
    out = tmp_path / "caller"
    subprocess.run(["g++", "-std=c++17", "-I", str(ROOT / "include"), "-I", CUDA_INC, str(src),
                    "-o", str(out), "-L", str(_lib.LIB_PATH.parent), "-lforgert_b200",
                    "-L/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{_lib.LIB_PATH.parent}"],
                   check=True)
    assert out.exists()


@pytest.mark.skipif(not (REF / "runtime" / "executor.cpp").exists(), reason="reference tree absent")
def test_reference_executor_compiles_unchanged_against_shim():
    """runtime/executor.cpp (which calls decode_attn_v4_flash at :165-170 and
    prefill_attn_causal at :158-163) compiles as-is with this repo's
    include/ ahead of the reference's kernels/ directory."""
    cmd = ["g++", "-std=c++17", "-fsyntax-only",
           "-I", str(ROOT / "include"),
           "-I", str(REF / "runtime" / "include"), "-I", str(REF / "kernels"), "-I", CUDA_INC,
           str(REF / "runtime" / "executor.cpp")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    # and the include really resolved to the drop-in, not the reference header
    r = subprocess.run(cmd[:-1] + ["-M", str(REF / "runtime" / "executor.cpp")], capture_output=True,
                       text=True)
    deps = r.stdout
    assert str(ROOT / "include" / "attention.cuh") in deps
    assert str(REF / "kernels" / "attention.cuh") not in deps


@pytest.mark.parametrize("env,want", [(None, 1000), ("60000", 5000), ("0", 1), ("250", 250)])
def test_exchange_wait_limit_is_capped(env, want):
    """FORGERT_EXCHANGE_WAIT_MS bounds the in-kernel spin on a peer's words;
    it is clamped to 1 ms .. 5 s (read once per process, so each value runs
    in a fresh process)."""
    import sys
    code = ("import sys; sys.path.insert(0, sys.argv[1]); from forgert_b200 import _lib; "
            "print(_lib.load().fr_exchange_wait_limit_ms())")
    e = dict(os.environ)
    e.pop("FORGERT_EXCHANGE_WAIT_MS", None)
    if env is not None:
        e["FORGERT_EXCHANGE_WAIT_MS"] = env
    r = subprocess.run([sys.executable, "-c", code, str(ROOT)], capture_output=True, text=True,
                       env=e, timeout=120)
    assert r.returncode == 0, r.stderr
    assert int(r.stdout.strip()) == want
