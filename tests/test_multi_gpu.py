"""Multi-GPU paths on real GPUs (NCCL), one process per GPU.

* Long context: the KV range of one sequence is split across the ranks; each
  rank computes its (m, l, acc) states with fr_decode_attn_partial, one NCCL
  all-gather exchanges them, fr_lse_merge_strided merges.  Every rank's
  output must match the CPU oracle over the whole range.
* Long context, exchange in the kernel: fr_decode_attn_exchange stores each
  rank's states into every rank's buffer (CUDA IPC mappings, plain peer
  stores) and merges what arrives; eager and CUDA-graph replays.
* Batched: (sequence, kv head) units are sharded by LPT; each rank decodes its
  own units from its own KV pool with no collective.  The outputs are
  gathered afterwards (verification only) and compared with the oracle.

Skipped when fewer than two GPUs are visible.  Ranks run as child processes
with a short process-group timeout, so a failing rank ends the test with an
error instead of a hang.
"""
from __future__ import annotations

import os
import socket
import traceback

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL, EPS = 2e-3, 1e-2, 1e-3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_q):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        from forgert_b200 import attention as A
        from forgert_b200 import sharding as SH
        from forgert_b200 import workloads as W
        from oracle import oracle as O

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        errs = {}

        # ---- long context: KV range split + all-gather of states + merge
        H, Hkv, D, T = 28, 4, 128, 20000
        q, k, v = W.decode_inputs(41, H, Hkv, D, T)
        b, e = SH.kv_ranges(T, world)[rank]
        dec = SH.LongContextDecoder(H, Hkv, D, dev)
        s = torch.cuda.Stream(dev)
        qd = torch.from_numpy(q).to(dev)
        kd = torch.from_numpy(np.ascontiguousarray(k[b:e])).to(dev)
        vd = torch.from_numpy(np.ascontiguousarray(v[b:e])).to(dev)
        out = torch.full((H, D), float("nan"), dtype=torch.float16, device=dev)
        with torch.cuda.stream(s):
            for _ in range(2):                       # twice: counters/workspace reused
                dec(qd, kd, vd, e - b, out, s)
        torch.cuda.synchronize()
        exact = O.decode_f64(q, k, v)
        errs["long"] = O.max_errors(out.cpu().numpy(), exact, EPS)

        # ---- long context, exchange inside the kernel (peer stores over NVLink)
        px = SH.PeerExchangeDecoder(H, Hkv, D, dev)
        outp = torch.full((H, D), float("nan"), dtype=torch.float16, device=dev)
        with torch.cuda.stream(s):
            for _ in range(3):                       # epochs 1..3: both buffer parities
                px(qd, kd, vd, e - b, outp, s)
        torch.cuda.synchronize()
        assert A.device_error() == 0
        errs["long_peer"] = O.max_errors(outp.cpu().numpy(), exact, EPS)
        # and as a CUDA graph, replayed
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            px(qd, kd, vd, e - b, outp, s)
        for _ in range(3):
            outp.fill_(float("nan"))
            g.replay()
        torch.cuda.synchronize()
        assert A.device_error() == 0
        errs["long_peer_graph"] = O.max_errors(outp.cpu().numpy(), exact, EPS)
        del g
        px.close()

        # ---- batched: units by LPT, own pool per rank, no collective
        rng = np.random.default_rng(42)
        B, H3, Hkv3, D3, G = 12, 28, 4, 128, 7
        lens = rng.integers(1, 3000, size=B).astype(np.int32)
        q3 = W.normal_fp16(rng, (B, H3, D3))
        ks = [W.normal_fp16(rng, (int(n), Hkv3, D3)) for n in lens]
        vs = [W.normal_fp16(rng, (int(n), Hkv3, D3)) for n in lens]
        mine = SH.shard_batched(lens, Hkv3, world)[rank]
        kpool = np.concatenate([ks[bb][:, h:h + 1] for bb, h, _ in mine])
        vpool = np.concatenate([vs[bb][:, h:h + 1] for bb, h, _ in mine])
        offs = np.concatenate([[0], np.cumsum([n for _, _, n in mine])[:-1]]).astype(np.int64)
        qu = np.stack([q3[bb, h * G:(h + 1) * G] for bb, h, _ in mine])
        ou = torch.full(qu.shape, float("nan"), dtype=torch.float16, device=dev)
        A.decode_attn_batched(torch.from_numpy(qu).to(dev), torch.from_numpy(kpool).to(dev),
                              torch.from_numpy(vpool).to(dev), torch.from_numpy(offs).to(dev),
                              torch.tensor([n for _, _, n in mine], dtype=torch.int32, device=dev),
                              ou, len(mine), G, 1, D3, kpool.shape[0],
                              int(max(n for _, _, n in mine)))
        torch.cuda.synchronize()
        full = torch.zeros((B, H3, D3), dtype=torch.float32, device=dev)
        for i, (bb, h, _) in enumerate(mine):
            full[bb, h * G:(h + 1) * G] = ou[i].float()
        dist.all_reduce(full)                        # verification only: disjoint slices
        errs["batched"] = O.max_errors(full.cpu().numpy(), O.batched_f64(q3, ks, vs, lens), EPS)
        assert A.device_error() == 0
        dist.barrier()
        dist.destroy_process_group()
        result_q.put((rank, errs, None))
    except Exception:
        result_q.put((rank, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_long_context_and_batched():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, errs, tb in results:
        assert tb is None, tb
        for name, (a, r) in errs.items():
            assert a <= ATOL and r <= RTOL, (rank, name, a, r)
