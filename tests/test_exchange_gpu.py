"""fr_decode_attn_exchange on one GPU: the in-kernel cross-GPU exchange of
split-KV states, in the forms a single GPU can run without one launch
waiting on another launch.

* world = 1: the kernel stores its state into its own buffer and merges it.
* world = 2 with the peer's part pre-written: rank 1's (m, l, acc) state of
  the second half of the range is written into rank 0's buffer as the tagged
  words rank 1 would store there over NVLink (call number << 32 | fp32
  bits); rank 0's call then merges both.  Two calls in a row exercise both
  buffer parities and the epoch advance.
* a peer that never arrives: the bounded wait ends after about a second,
  the device error word reads "peer timeout", the context stays usable and
  fr_exchange_reset makes the buffer usable again.

Outputs are compared with the fp64 oracle at max |x - r| <= 2e-3 and
max |x - r| / max(|r|, 1e-3) <= 1e-2.  The two-GPU form runs in
tests/test_multi_gpu.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from forgert_b200 import attention as A
from forgert_b200 import workloads as W
from oracle import oracle as O

from test_decode_gpu import assert_close, dev, nan_like

pytestmark = pytest.mark.gpu

DEV_TIMEOUT_PEER = 3


def new_buffer(H, D, world):
    lay = A.exchange_layout(H, D, world)
    return torch.zeros(lay["bytes"] // 4, dtype=torch.float32, device="cuda"), lay


@pytest.mark.parametrize("H,Hkv,D,T", [(28, 4, 128, 20000), (12, 2, 128, 700), (14, 2, 64, 1)])
def test_exchange_single_rank(H, Hkv, D, T):
    q, k, v = W.decode_inputs(50 + T, H, Hkv, D, T)
    exact = O.decode_f64(q, k, v)
    buf, _ = new_buffer(H, D, 1)
    qd, kd, vd = dev(q), dev(k), dev(v)
    for _ in range(3):                               # epochs 1..3, both parities
        out = nan_like(qd)
        A.decode_attn_exchange(qd, kd, vd, T, out, H, Hkv, D, [buf], 0, 1)
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert_close(out.cpu().numpy(), exact, what=f"exchange world=1 T={T}")
    assert int(buf.view(torch.int32)[0]) == 3          # epoch advanced once per call


def test_exchange_single_rank_graph_replays():
    H, Hkv, D, T = 28, 4, 128, 5000
    q, k, v = W.decode_inputs(61, H, Hkv, D, T)
    exact = O.decode_f64(q, k, v)
    buf, _ = new_buffer(H, D, 1)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = nan_like(qd)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        A.decode_attn_exchange(qd, kd, vd, T, out, H, Hkv, D, [buf], 0, 1, stream=s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        A.decode_attn_exchange(qd, kd, vd, T, out, H, Hkv, D, [buf], 0, 1, stream=s)
    for _ in range(4):
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert_close(out.cpu().numpy(), exact, what="exchange graph replay")
    assert int(buf.view(torch.int32)[0]) == 5


def tagged(values: torch.Tensor, epoch: int) -> torch.Tensor:
    """fp32 values as exchange words: (epoch << 32) | bits."""
    bits = values.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return bits | (epoch << 32)


@pytest.mark.parametrize("H,Hkv,D,T,split", [(28, 4, 128, 30000, 14976), (12, 2, 64, 513, 0)])
def test_exchange_two_ranks_with_prewritten_peer(H, Hkv, D, T, split):
    """Rank 0 holds rows [0, split), 'rank 1' rows [split, T) (split 0: rank 0 empty)."""
    q, k, v = W.decode_inputs(70 + T, H, Hkv, D, T)
    exact = O.decode_f64(q, k, v)
    buf0, lay = new_buffer(H, D, 2)
    buf1, _ = new_buffer(H, D, 2)                     # stands in for rank 1's buffer
    w0, w1 = buf0.view(torch.int64), buf1.view(torch.int64)
    qd = dev(q)
    k0, v0 = dev(k[:split]) if split else None, dev(v[:split]) if split else None
    k1, v1 = dev(k[split:]), dev(v[split:])
    ml1 = torch.empty((H, 2), dtype=torch.float32, device="cuda")
    acc1 = torch.empty((H, D), dtype=torch.float32, device="cuda")
    A.decode_attn_partial(qd, k1, v1, T - split, ml1, acc1, H, Hkv, D)
    for epoch in (1, 2):
        par = epoch & 1
        ml_off = lay["ml"] // 8 + (par * 2 + 1) * H * 2
        acc_off = lay["acc"] // 8 + (par * 2 + 1) * H * D
        w0[ml_off:ml_off + H * 2].copy_(tagged(ml1.view(-1), epoch))
        w0[acc_off:acc_off + H * D].copy_(tagged(acc1.view(-1), epoch))
        out = nan_like(qd)
        A.decode_attn_exchange(qd, k0, v0, split, out, H, Hkv, D, [buf0, buf1], 0, 2)
        torch.cuda.synchronize()
        assert A.device_error() == 0
        assert_close(out.cpu().numpy(), exact, what=f"exchange world=2 epoch {epoch}")
        assert int(buf0.view(torch.int32)[0]) == epoch
    # rank 0 also stored its own state into 'rank 1's' buffer: parity 0, source 0,
    # tagged with call 2
    own = w1[lay["acc"] // 8: lay["acc"] // 8 + H * D]
    assert bool(((own >> 32) == 2).all())


def test_exchange_peer_timeout_is_reported_and_recoverable():
    H, Hkv, D, T = 12, 2, 128, 256
    q, k, v = W.decode_inputs(90, H, Hkv, D, T)
    buf0, lay = new_buffer(H, D, 2)
    buf1, _ = new_buffer(H, D, 2)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = nan_like(qd)
    A.decode_attn_exchange(qd, kd, vd, T, out, H, Hkv, D, [buf0, buf1], 0, 2)  # nobody is rank 1
    torch.cuda.synchronize()
    assert A.device_error(clear=True) == DEV_TIMEOUT_PEER
    # the context is fine: reset the buffer and run a complete single-rank call
    lib = A.load()
    assert lib.fr_exchange_reset(buf0.data_ptr(), lay["bytes"], None) == 0
    buf, _ = new_buffer(H, D, 1)
    A.decode_attn_exchange(qd, kd, vd, T, out, H, Hkv, D, [buf], 0, 1)
    torch.cuda.synchronize()
    assert A.device_error() == 0
    assert_close(out.cpu().numpy(), O.decode_f64(q, k, v), what="after timeout")
    assert int(buf0.view(torch.int32)[0]) == 0 and not bool(buf0.view(torch.int64).any())
