"""Multi-GPU partitioning logic, run as gloo ranks on CPU.

The device kernels are replaced by the numpy oracle; what is under test is
the host side: unit assignment, KV-range cuts, the one all-gather of packed
(m, l, acc) states and the merge over the gathered buffer.  A rank that fails
before the exchange is detected by the others through the process group's
timeout (no GPU involved).
"""
from __future__ import annotations

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from forgert_b200 import sharding as SH
from forgert_b200 import workloads as W
from oracle import oracle as O


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# ------------------------------------------------------------ pure host logic
def test_lpt_assign_balances_and_covers():
    lens = W.cfg3_lens()
    for world in (1, 2, 4, 8):
        shards = SH.shard_batched(lens, 4, world)
        units = sorted(u for s in shards for u in s)
        assert units == sorted(SH.batched_units(lens, 4))      # every unit exactly once
        loads = [sum(u[2] for u in s) for s in shards]
        assert max(loads) - min(loads) <= 8192                  # LPT bound: one largest unit
        assert max(loads) / (sum(loads) / world) < 1.02
    assert SH.lpt_assign([5, 5, 5], 2) == SH.lpt_assign([5, 5, 5], 2)   # deterministic


def test_kv_ranges_cover_and_align():
    for kv, world in [(131072, 8), (131072, 3), (100, 4), (1, 2), (0, 2), (4097, 2)]:
        rs = SH.kv_ranges(kv, world)
        assert len(rs) == world
        assert rs[0][0] == 0 and rs[-1][1] == kv
        for (b0, e0), (b1, _) in zip(rs, rs[1:]):
            assert e0 == b1
        for b, e in rs:
            assert (b % 64 == 0 or b == kv) and e >= b
        sizes = [e - b for b, e in rs]
        assert max(sizes) - min(sizes) <= 2 * 64 or kv < 64 * world   # one tile + the ragged tail


# ---------------------------------------------------------- gloo rank bodies
def _np_partial(q, k_local, v_local, local_len, ml, acc):
    m, l, a = O.partial_f64(q.numpy(), k_local.numpy(), v_local.numpy(), 0, local_len)
    ml[:, 0] = torch.from_numpy(m)
    ml[:, 1] = torch.from_numpy(l)
    acc.copy_(torch.from_numpy(a))


def _np_merge(H, D):
    def merge(gathered, world, out):
        g = gathered.numpy()
        ml = g[:, :2 * H].reshape(world, H, 2)
        acc = g[:, 2 * H:].reshape(world, H, D)
        out.copy_(torch.from_numpy(O.merge_f64(ml[..., 0], ml[..., 1], acc)))
    return merge


def _long_context_rank(rank, world, port, result_q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        H, Hkv, D, T = 28, 4, 128, 3000
        q, k, v = W.decode_inputs(3, H, Hkv, D, T)        # every rank draws the same full problem
        b, e = SH.kv_ranges(T, world)[rank]               # ... and keeps only its range
        dec = SH.LongContextDecoder(H, Hkv, D, "cpu", partial_fn=_np_partial,
                                    merge_fn=_np_merge(H, D))
        out = torch.zeros((H, D), dtype=torch.float64)
        dec(torch.from_numpy(q), torch.from_numpy(k[b:e]), torch.from_numpy(v[b:e]), e - b, out)
        err = float(np.abs(out.numpy() - O.decode_f64(q, k, v)).max())
        result_q.put((rank, err, None))
        dist.destroy_process_group()
    except Exception:
        result_q.put((rank, None, traceback.format_exc()))


def _batched_rank(rank, world, port, result_q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(12)
        B, H, Hkv, D = 6, 28, 4, 64
        lens = rng.integers(1, 400, size=B)
        q = W.normal_fp16(rng, (B, H, D))
        ks = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
        vs = [W.normal_fp16(rng, (int(n), Hkv, D)) for n in lens]
        G = H // Hkv
        out = torch.zeros((B, H, D), dtype=torch.float64)
        mine = SH.shard_batched(lens, Hkv, world)[rank]
        for b, h, n in mine:                              # only this rank's units
            qs = q[b, h * G:(h + 1) * G]
            out[b, h * G:(h + 1) * G] = torch.from_numpy(
                O.decode_f64(qs, ks[b][:, h:h + 1], vs[b][:, h:h + 1]))
        # verification only (not part of the decode path): sum the disjoint slices
        dist.all_reduce(out)
        err = float(np.abs(out.numpy() - O.batched_f64(q, ks, vs, lens)).max())
        result_q.put((rank, err, None))
        dist.destroy_process_group()
    except Exception:
        result_q.put((rank, None, traceback.format_exc()))


def _run(body, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=body, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("world", [2])
def test_long_context_gloo(world):
    for rank, err, tb in _run(_long_context_rank, world):
        assert tb is None, tb
        assert err < 1e-6, (rank, err)       # states cross the exchange as fp32


def test_batched_sharding_gloo():
    for rank, err, tb in _run(_batched_rank, 2):
        assert tb is None, tb
        assert err < 1e-12, (rank, err)


def _dropout_rank(rank, world, port, result_q):
    """Rank 1 fails before the exchange; rank 0 must get an error, not hang."""
    from datetime import timedelta
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        if rank == 1:
            result_q.put((rank, "left", None))
            result_q.close()
            result_q.join_thread()                        # flush before the abrupt exit
            os._exit(0)                                   # leaves between steps, nothing in flight
        dec = SH.LongContextDecoder(8, 2, 64, "cpu", partial_fn=_np_partial,
                                    merge_fn=_np_merge(8, 64))
        q, k, v = W.decode_inputs(1, 8, 2, 64, 100)
        try:
            dec(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), 100,
                torch.zeros((8, 64), dtype=torch.float64))
            result_q.put((rank, "no error", None))
        except Exception as e:                            # the collective fails with an error
            result_q.put((rank, "error", type(e).__name__))
    except Exception:
        result_q.put((rank, None, traceback.format_exc()))


def test_rank_failure_surfaces_as_error():
    res = dict((r, (s, x)) for r, s, x in _run(_dropout_rank, 2))
    assert res[1][0] == "left"
    assert res[0][0] == "error", res[0]
