"""fr_copy_async: stream-ordered kernel copies between device memory and
page-locked host memory, bit-exact, at aligned and unaligned sizes and
offsets, under CUDA-graph capture, and chained with a decode call the way a
decode step stages its inputs and outputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from forgert_b200._lib import ForgeRTError
from oracle import oracle as O

from test_decode_gpu import assert_close

pytestmark = pytest.mark.gpu

SIZES = [1, 15, 16, 17, 4096, 86016, (1 << 20) + 3]


def pattern(n: int, seed: int) -> torch.Tensor:
    return torch.from_numpy(np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8))


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("direction", ["h2d", "d2h", "d2d"])
def test_copy_exact(n, direction):
    src_cpu = pattern(n, n)
    if direction == "h2d":
        src, dst = src_cpu.pin_memory(), torch.zeros(n, dtype=torch.uint8, device="cuda")
    elif direction == "d2h":
        src, dst = src_cpu.cuda(), torch.zeros(n, dtype=torch.uint8).pin_memory()
    else:
        src, dst = src_cpu.cuda(), torch.zeros(n, dtype=torch.uint8, device="cuda")
    A.copy_async(dst, src)
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu(), src_cpu)


@pytest.mark.parametrize("off_src,off_dst", [(1, 0), (0, 3), (5, 5), (16, 32)])
def test_copy_unaligned_offsets(off_src, off_dst):
    n = 10007
    base = pattern(n + 64, 7)
    src = base.pin_memory()
    dst = torch.zeros(n + 64, dtype=torch.uint8, device="cuda")
    A.copy_async(dst.data_ptr() + off_dst, src.data_ptr() + off_src, n)
    torch.cuda.synchronize()
    got = dst.cpu()
    assert torch.equal(got[off_dst:off_dst + n], base[off_src:off_src + n])
    assert not bool(got[:off_dst].any()) and not bool(got[off_dst + n:].any())


def test_copy_zero_bytes_and_pageable_host():
    d = torch.zeros(16, dtype=torch.uint8, device="cuda")
    A.copy_async(d, torch.ones(16, dtype=torch.uint8).pin_memory(), 0)
    torch.cuda.synchronize()
    assert not bool(d.any())
    pageable = np.ones(16, dtype=np.uint8)
    with pytest.raises(ForgeRTError):
        A.copy_async(d.data_ptr(), pageable.ctypes.data, 16)


def test_copy_in_graph_with_decode_step():
    """copy q in -> fr_decode_attn -> copy out, captured once and replayed
    with new host contents each time (the bench's e2e structure)."""
    H, Hkv, D, T = 12, 2, 128, 3000
    rng = np.random.default_rng(31)
    k = W.normal_fp16(rng, (T, Hkv, D))
    v = W.normal_fp16(rng, (T, Hkv, D))
    kd, vd = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    q_host = torch.empty((H, D), dtype=torch.float16).pin_memory()
    out_host = torch.empty((H, D), dtype=torch.float16).pin_memory()
    q_dev = torch.empty((H, D), dtype=torch.float16, device="cuda")
    out_dev = torch.empty_like(q_dev)
    s = torch.cuda.Stream()

    def body(st):
        A.copy_async(q_dev, q_host, stream=st)
        A.decode_attn_v4_flash(q_dev, kd, vd, out_dev, H, Hkv, D, T, st)
        A.copy_async(out_host, out_dev, stream=st)

    q_host.copy_(torch.from_numpy(W.normal_fp16(rng, (H, D))))
    with torch.cuda.stream(s):
        body(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        body(torch.cuda.current_stream())
    for i in range(3):
        q = W.normal_fp16(rng, (H, D))
        q_host.copy_(torch.from_numpy(q))
        out_host.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert_close(out_host.numpy(), O.decode_f64(q, k, v), what=f"graph replay {i}")
