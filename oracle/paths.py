"""Where the parity checkers find the reference sources and their headers.

TEST INFRASTRUCTURE ONLY (used by oracle/Makefile's callers, tests/ and
tests/golden/make_golden.py).  Nothing names a machine path:

reference_tree()    FORGERT_REFERENCE_TREE, else BASELINE.json's
                    "reference_path"; None when that directory is absent
                    (e.g. on a GPU box, which only uses the prebuilt
                    oracle/_ref files).
json_include_dir()  FORGERT_JSON_INCLUDE, else the directory of this Python
                    installation's site-packages that holds
                    nlohmann/json.hpp (the reference's runtime needs it and
                    does not vendor it); None when there is none.
"""
from __future__ import annotations

import json
import os
import sysconfig
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def reference_tree() -> Path | None:
    p = os.environ.get("FORGERT_REFERENCE_TREE")
    if not p:
        try:
            p = json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            p = None
    return Path(p) if p and Path(p).is_dir() else None


def json_include_dir() -> Path | None:
    p = os.environ.get("FORGERT_JSON_INCLUDE")
    if p:
        return Path(p) if (Path(p) / "nlohmann" / "json.hpp").exists() else None
    patterns = ("include/nlohmann/json.hpp", "include/*/thirdparty/nlohmann/json.hpp",
                "*/include/nlohmann/json.hpp", "*/include/*/thirdparty/nlohmann/json.hpp",
                "*/thirdparty/nlohmann/json.hpp")
    for key in ("purelib", "platlib"):
        base = Path(sysconfig.get_paths()[key])
        for pat in patterns:
            for hit in sorted(base.glob(pat)):
                return hit.parent.parent
    return None


def make_args() -> list[str]:
    """REF=/JSON_DIR= arguments for `make -C oracle` (REF points nowhere when
    the reference tree is absent, which skips the reference builds)."""
    ref = reference_tree()
    args = [f"REF={ref}" if ref else "REF=/nonexistent"]
    inc = json_include_dir()
    if inc:
        args.append(f"JSON_DIR={inc}")
    return args
