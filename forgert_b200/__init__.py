"""forgert_b200 - B200-native (sm_100a) flash-decode attention for ForgeRT.

The compute path is libforgert_b200.so (hand-written CUDA, C ABI in
include/forgert_attn.h).  This package only mirrors the reference's launcher
interface on the host and generates the synthetic benchmark workloads.
"""
from ._lib import LIB_PATH, ForgeRTError  # noqa: F401

__version__ = "0.1.0"
