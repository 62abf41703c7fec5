#!/usr/bin/env python
"""Decode-attention benchmark (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload cfg2|cfg3|cfg3p|cfg4]

Default workload (cfg2, the configuration the headline metric is quoted on):
Qwen2-1.5B-shaped decode attention, batch 1, 12 query heads, 2 KV heads,
head_dim 128, over all 28 layers of a contiguous fp16 cache
[28 x 2 x 16384 x 2 x 128] (470 MB, N(0,1) synthetic data), once at each
kv_len in {512, 2048, 4096, 16384}.  One step = those 4 x 28 = 112
decode_attn_v4_flash-equivalent calls (fr_decode_attn).  Each kv_len group
is one CUDA graph of 28 calls; L2 is flushed (256 MiB write) before every
group and the CUDA events bracket only the group, so every K/V byte comes
from HBM.  metric = algorithmic bytes (K+V of the valid range + q + out)
per second.

With N > 1 (torchrun) every rank decodes its own sequence (its own cache,
seeded by rank): batched decode sharded by sequence, no collective on the
data path; value = all ranks' bytes / the slowest rank's time ("weak").

--workload cfg3 (batched ragged, 64 sequences x 4 kv heads sharded by
(sequence, kv head) across ranks, "strong") and cfg4 (one 128K-token
sequence, KV range split across ranks, NCCL all-gather of the per-rank
(m, l, acc) states + LSE merge, "strong") measure the multi-GPU paths.
--workload cfg3p is cfg3 in a paged KV cache (16-row pages in shuffled order,
one block table per sequence, fr_decode_attn_paged), sharded by sequence.

--impl reference times the reference's own CPU implementation
(cpu_decode_attn, tests/test_kernels.cpp:229-270, compiled from the
reference sources into oracle/_ref) on the same workload with all host
threads; rank 0 alone runs it.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from forgert_b200 import workloads as W  # noqa: E402

METRIC = "decode-attn HBM GB/s (algorithmic K+V+q+out bytes / s)"
UNIT = "GB/s"
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours",
                    help="reference = the reference's CPU implementation")
    ap.add_argument("--workload", choices=["cfg2", "cfg3", "cfg3p", "cfg4"], default="cfg2")
    ap.add_argument("--page-size", type=int, default=16, help="cfg3p page rows (multiple of 16)")
    ap.add_argument("--page-order", choices=["shuffled", "sequential"], default="shuffled",
                    help="cfg3p: pages handed out in a seeded random order, or in order")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="cfg4 at N > 1: in-kernel peer exchange or NCCL all-gather")
    ap.add_argument("--layers", type=int, default=1,
                    help="cfg4: layer caches decoded back to back per step (default 1 call)")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of graphs")
    ap.add_argument("--no-overlap", action="store_true",
                    help="disable launch overlap (pre-wait K/V prefetch under PDL)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling run: few steps, no clocks/e2e/cpu legs")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def emit(obj) -> None:
    print(json.dumps(obj), flush=True)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_per_launch():
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except Exception:
        return None


# ------------------------------------------------------------ clock sampler
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every few ms."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.samples = []
        self.period = period_s
        self.stop_ev = threading.Event()
        self.ok = False
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = self._handle(pynvml, torch, cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.ok = True
        except Exception:
            self.nvml = None
        self.t = threading.Thread(target=self._run, daemon=True)

    @staticmethod
    def _handle(pynvml, torch, cuda_index):
        """NVML handle of the CUDA device (matched by PCI bus id when possible)."""
        try:
            p = torch.cuda.get_device_properties(cuda_index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            ids = [v for v in vis.split(",") if v.strip().isdigit()]
            idx = int(ids[cuda_index]) if cuda_index < len(ids) else cuda_index
            return pynvml.nvmlDeviceGetHandleByIndex(idx)

    def _run(self):
        n = self.nvml
        while not self.stop_ev.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)
                rs = self.reasons_fn(self.h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t.start()
        return self

    def __exit__(self, *a):
        self.stop_ev.set()
        if self.ok:
            self.t.join(timeout=2)

    def summary(self):
        if not self.ok or not self.samples:
            return None
        mhz = [s[0] for s in self.samples]
        mask = 0
        for _, r in self.samples:
            mask |= int(r)
        reasons = [name for bit, name in self.REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


# --------------------------------------------------------------- our arm
class Cfg2:
    """28 layers x kv_len {512, 2048, 4096, 16384}, one sequence per rank."""

    L, S, H, HKV, D = W.CFG2_LAYERS, W.CFG2_MAX_SEQ, 12, 2, 128

    def __init__(self, torch, rank: int, device):
        self.torch = torch
        g = torch.Generator(device=device)
        g.manual_seed(1 + 1000 * rank)
        self.cache = torch.empty((self.L, 2, self.S, self.HKV, self.D), dtype=torch.float16,
                                 device=device)
        self.cache.normal_(generator=g)
        self.q = torch.empty((self.L, self.H, self.D), dtype=torch.float16, device=device)
        self.q.normal_(generator=g)
        self.out = torch.empty_like(self.q)
        self.groups = list(W.CFG2_KV_LENS)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()

    def bytes_per_group(self, kv: int) -> int:
        return self.L * W.decode_bytes([kv], self.H, self.HKV, self.D)

    def bytes_per_step(self) -> int:
        return sum(self.bytes_per_group(kv) for kv in self.groups)

    def calls_per_group(self) -> int:
        return self.L

    def workspace_bytes(self, A) -> int:
        return max(A.decode_workspace_size(1, self.H, self.HKV, self.D, kv) for kv in self.groups)

    def run_group(self, A, kv: int, stream) -> None:
        for l in range(self.L):
            A.decode_attn_v4_flash(self.q[l], self.cache[l, 0], self.cache[l, 1], self.out[l],
                                   self.H, self.HKV, self.D, kv, stream)

    def e2e_bytes(self):
        per = self.H * self.D * 2
        n = self.L * len(self.groups)
        return n * per, n * per

    scaling = "weak"
    graphable = True

    def call_bytes(self, kv: int) -> int:
        return W.decode_bytes([kv], self.H, self.HKV, self.D)

    def config(self):
        return {
            "workload": "cfg2: Qwen2-1.5B-shape decode attention, batch 1 per GPU, "
                        "28 layers x kv_len {512, 2048, 4096, 16384}",
            "shape": "Qwen2-1.5B attention (H12, Hkv2, D128), random data",
            "batch_per_gpu": 1, "num_heads": self.H, "num_kv_heads": self.HKV,
            "head_dim": self.D, "layers": self.L, "kv_lens": self.groups,
            "cache": "contiguous fp16 [28 x 2 x 16384 x 2 x 128] per GPU",
            "l2": "flushed (256 MiB write) before each kv_len group; events exclude the flush",
        }


class Cfg3:
    """Qwen2-7B batched decode: 64 sequences, kv_len ~ U{1024..8192} (seed 2),
    H28 Hkv4 D128.  The 256 (sequence, kv head) units are assigned to ranks
    by LPT on token count; each rank keeps its units in one KV pool
    [rows, 1, 128] (a unit is one kv head with its 7 query heads) and runs one
    batched call.  Total work is fixed ("strong")."""

    H, HKV, D, G = 28, 4, 128, 7
    scaling = "strong"
    graphable = True

    def __init__(self, torch, rank: int, world: int, device):
        from forgert_b200 import sharding as SH
        self.torch = torch
        self.lens_all = W.cfg3_lens()
        mine = SH.shard_batched(self.lens_all, self.HKV, world)[rank]
        self.units = mine
        lens = [u[2] for u in mine]
        self.U = len(mine)
        rows = int(sum(lens))
        offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        g = torch.Generator(device=device)
        g.manual_seed(2 + 1000 * rank)
        self.kpool = torch.empty((rows, 1, self.D), dtype=torch.float16, device=device).normal_(generator=g)
        self.vpool = torch.empty((rows, 1, self.D), dtype=torch.float16, device=device).normal_(generator=g)
        self.offs = torch.from_numpy(offs).to(device)
        self.lens = torch.tensor(lens, dtype=torch.int32, device=device)
        self.q = torch.empty((self.U, self.G, self.D), dtype=torch.float16, device=device).normal_(generator=g)
        self.out = torch.empty_like(self.q)
        self.rows = rows
        self.max_len = int(max(lens))
        self.groups = ["batch"]
        self.my_bytes = W.decode_bytes(lens, self.G, 1, self.D)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()

    def bytes_per_group(self, key) -> int:
        return self.my_bytes

    def bytes_per_step(self) -> int:
        return self.my_bytes

    def job_bytes(self) -> int:
        return W.decode_bytes(self.lens_all, self.H, self.HKV, self.D)

    def call_bytes(self, key) -> int:
        return self.my_bytes

    def calls_per_group(self) -> int:
        return 1

    def workspace_bytes(self, A) -> int:
        return A.decode_workspace_size(self.U, self.G, 1, self.D, self.max_len)

    def run_group(self, A, key, stream) -> None:
        A.decode_attn_batched(self.q, self.kpool, self.vpool, self.offs, self.lens, self.out,
                              self.U, self.G, 1, self.D, self.rows, self.max_len, stream)

    def e2e_bytes(self):
        n = self.U * self.G * self.D * 2
        return n, n

    def config(self):
        return {
            "workload": "cfg3: Qwen2-7B-shape batched decode attention, 64 sequences, ragged "
                        "kv_len U{1024..8192} (seed 2), sharded by (sequence, kv head)",
            "shape": "Qwen2-7B attention (H28, Hkv4, D128), random data",
            "global_batch": 64, "num_heads": self.H, "num_kv_heads": self.HKV,
            "head_dim": self.D, "total_kv_tokens": int(self.lens_all.sum()),
            "units_this_rank": self.U,
            "l2": "flushed (256 MiB write) before each call; events exclude the flush",
        }


class Cfg3Paged(Cfg3):
    """cfg3's 64 sequences in a paged KV cache: pages of page_size rows x 4 kv heads
    x 128, handed out in a seeded random order (a fragmented serving cache),
    one block table per sequence, one fr_decode_attn_paged call.  N GPUs:
    whole sequences are assigned by LPT on length; no collective."""

    def __init__(self, torch, rank: int, world: int, device, page_size: int = 16,
                 page_order: str = "shuffled"):
        from forgert_b200 import sharding as SH
        self.torch = torch
        self.PAGE = page_size
        self.lens_all = W.cfg3_lens()
        mine = SH.lpt_assign(self.lens_all, world)[rank]
        lens = [int(self.lens_all[i]) for i in mine]
        self.B = len(mine)
        need = [-(-n // self.PAGE) for n in lens]
        self.num_pages = int(sum(need))
        width = max(need)
        self.page_order = page_order
        order = (np.random.default_rng(5 + rank).permutation(self.num_pages)
                 if page_order == "shuffled" else np.arange(self.num_pages))
        table = np.full((self.B, width), -1, np.int32)
        o = 0
        for b, n in enumerate(need):
            table[b, :n] = order[o:o + n]
            o += n
        g = torch.Generator(device=device)
        g.manual_seed(2 + 1000 * rank)
        shape = (self.num_pages, self.PAGE, self.HKV, self.D)
        self.kpages = torch.empty(shape, dtype=torch.float16, device=device).normal_(generator=g)
        self.vpages = torch.empty(shape, dtype=torch.float16, device=device).normal_(generator=g)
        self.table = torch.from_numpy(table).to(device)
        self.width = width
        self.lens = torch.tensor(lens, dtype=torch.int32, device=device)
        self.q = torch.empty((self.B, self.H, self.D), dtype=torch.float16, device=device).normal_(generator=g)
        self.out = torch.empty_like(self.q)
        self.max_len = int(max(lens))
        self.groups = ["batch"]
        self.my_bytes = W.decode_bytes(lens, self.H, self.HKV, self.D)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()
        self.U = self.B

    def workspace_bytes(self, A) -> int:
        return A.decode_workspace_size(self.B, self.H, self.HKV, self.D, self.max_len)

    def run_group(self, A, key, stream) -> None:
        A.decode_attn_paged(self.q, self.kpages, self.vpages, self.table, self.lens, self.out,
                            self.B, self.H, self.HKV, self.D, self.PAGE, self.num_pages,
                            self.width, self.max_len, stream)

    def e2e_bytes(self):
        n = self.B * self.H * self.D * 2
        return n, n

    def config(self):
        c = super().config()
        c["workload"] = (f"cfg3p: cfg3's 64 sequences in a paged KV cache ({self.PAGE}-row pages in "
                         f"{self.page_order} order, block table per sequence), sharded by sequence")
        c.pop("units_this_rank", None)
        c.update({"page_size": self.PAGE, "page_order": self.page_order,
                  "sequences_this_rank": self.B,
                  "num_pages_this_rank": self.num_pages})
        return c


class Cfg4:
    """Qwen2-7B long context: one sequence, kv_len 131072, H28 Hkv4 D128.
    One GPU: a plain fr_decode_attn call.  N GPUs: each rank holds a
    contiguous KV range.  exchange "peer" (default): one
    fr_decode_attn_exchange kernel per rank computes its states, stores them
    into every rank's exchange buffer over NVLink and merges what arrives;
    exchange "nccl": partial kernel, NCCL all-gather of the states, merge
    kernel.  `layers` > 1 runs that many layer caches back to back in one
    CUDA graph (a decode step's attention calls) instead of a single call.
    Total work is fixed ("strong")."""

    H, HKV, D, T = 28, 4, 128, 131072
    scaling = "strong"

    def __init__(self, torch, rank: int, world: int, device, exchange: str = "peer",
                 layers: int = 1):
        from forgert_b200 import sharding as SH
        self.torch = torch
        self.world = world
        self.L = max(1, layers)
        b, e = SH.kv_ranges(self.T, world)[rank]
        self.n = e - b
        g = torch.Generator(device=device)
        g.manual_seed(3 + 1000 * rank)
        self.k = torch.empty((self.L, max(self.n, 1), self.HKV, self.D), dtype=torch.float16,
                             device=device).normal_(generator=g)
        self.v = torch.empty_like(self.k).normal_(generator=g)
        self.q = torch.empty((self.L, self.H, self.D), dtype=torch.float16, device=device)
        self.q.normal_(generator=torch.Generator(device=device).manual_seed(33))
        self.out = torch.empty_like(self.q)
        self.groups = ["step"]
        self.exchange = exchange if world > 1 else "none"
        self.align_ranks = world > 1
        if world == 1:
            self.dec = None
        elif exchange == "peer":
            self.dec = SH.PeerExchangeDecoder(self.H, self.HKV, self.D, device)
        else:
            # the NCCL all-gather is captured in the same CUDA graph as the
            # partial and merge kernels (graphs are released before the
            # process group is destroyed)
            self.dec = SH.LongContextDecoder(self.H, self.HKV, self.D, device)
        self.graphable = True
        self.my_bytes = W.decode_bytes([self.n], self.H, self.HKV, self.D)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()

    def bytes_per_group(self, key) -> int:
        return self.my_bytes * self.L

    def bytes_per_step(self) -> int:
        return self.my_bytes * self.L

    def job_bytes(self) -> int:
        return W.decode_bytes([self.T], self.H, self.HKV, self.D) * self.L

    def call_bytes(self, key) -> int:
        return self.my_bytes

    def calls_per_group(self) -> int:
        return self.L

    def workspace_bytes(self, A) -> int:
        return A.decode_workspace_size(1, self.H, self.HKV, self.D, max(self.n, 1))

    def run_group(self, A, key, stream) -> None:
        for l in range(self.L):
            if self.dec is None:
                A.decode_attn_v4_flash(self.q[l], self.k[l], self.v[l], self.out[l], self.H,
                                       self.HKV, self.D, self.n, stream)
            else:
                self.dec(self.q[l], self.k[l], self.v[l], self.n, self.out[l], stream)

    def e2e_bytes(self):
        n = self.L * self.H * self.D * 2
        return n, n

    def config(self):
        return {
            "workload": "cfg4: Qwen2-7B-shape long-context decode attention, 1 sequence, "
                        "kv_len 131072, KV range split across GPUs, (m, l, acc) states "
                        "exchanged and merged",
            "exchange": {"none": "single GPU", "peer": "in-kernel peer stores over NVLink + "
                         "merge (fr_decode_attn_exchange)", "nccl": "NCCL all-gather + merge "
                         "kernel"}[self.exchange],
            "shape": "Qwen2-7B attention (H28, Hkv4, D128), random data",
            "global_batch": 1, "num_heads": self.H, "num_kv_heads": self.HKV,
            "head_dim": self.D, "kv_len": self.T, "kv_rows_this_rank": self.n,
            "layers": self.L,
            "l2": "flushed (256 MiB write) before each step; events exclude the flush",
            "rank_alignment": "N > 1: one-element NCCL all-reduce after the flush, before "
                              "the events (ranks start each call together)",
        }


def run_ours(args, torch, dist, rank, local_rank, world):
    from forgert_b200 import attention as A
    from forgert_b200 import _lib

    lib = _lib.load()
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if args.workload == "cfg2":
        wl = Cfg2(torch, rank, device)
    elif args.workload == "cfg3":
        wl = Cfg3(torch, rank, world, device)
    elif args.workload == "cfg3p":
        wl = Cfg3Paged(torch, rank, world, device, args.page_size, args.page_order)
    else:
        wl = Cfg4(torch, rank, world, device, args.exchange, args.layers)
    stream = torch.cuda.Stream(device)
    # Decode-step launch overlap: the attention kernel may stream K/V rows
    # older than the newest one while the preceding kernel finishes.
    lib.fr_set_launch_overlap(0 if args.no_overlap else 1)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    A.reserve_workspace(wl.workspace_bytes(A))
    torch.cuda.synchronize()

    # Eager warm-up (creates the library's device state outside capture).
    with torch.cuda.stream(stream):
        for kv in wl.groups:
            wl.run_group(A, kv, stream)
    torch.cuda.synchronize()

    use_graph = not args.no_graph and wl.graphable
    graphs = {}
    launches_per_step = 0
    if use_graph:
        for kv in wl.groups:
            g = torch.cuda.CUDAGraph()
            c0 = lib.fr_launch_count()
            with torch.cuda.graph(g, stream=stream):
                wl.run_group(A, kv, torch.cuda.current_stream())
            launches_per_step += lib.fr_launch_count() - c0
            graphs[kv] = g
    else:
        c0 = lib.fr_launch_count()
        with torch.cuda.stream(stream):
            for kv in wl.groups:
                wl.run_group(A, kv, stream)
        torch.cuda.synchronize()
        launches_per_step = lib.fr_launch_count() - c0

    # Workloads whose ranks exchange data inside the timed call (cfg4 at N > 1)
    # start each call together: a one-element all-reduce after the flush,
    # outside the events, so the per-rank flush and launch skew is not timed
    # as waiting for the slowest rank.
    align = torch.zeros(1, dtype=torch.float32, device=device) \
        if world > 1 and getattr(wl, "align_ranks", False) else None

    def step(events):
        for i, kv in enumerate(wl.groups):
            flush.fill_(i & 0xFF)
            if align is not None:
                dist.all_reduce(align)
            if events is not None:
                events[i][0].record(stream)
            if use_graph:
                graphs[kv].replay()
            else:
                wl.run_group(A, kv, stream)
            if events is not None:
                events[i][1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step(None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    K = args.steps
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in wl.groups]
          for _ in range(K)]
    sampler = ClockSampler(local_rank) if not args.ncu else None
    if sampler:
        sampler.__enter__()
    with torch.cuda.stream(stream):
        for k in range(K):
            step(ev[k])
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    group_ms = {kv: sum(ev[k][i][0].elapsed_time(ev[k][i][1]) for k in range(K))
                for i, kv in enumerate(wl.groups)}
    total_ms = sum(group_ms.values())
    assert A.device_error() == 0, "in-kernel wait timed out"
    max_ms = total_ms
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        max_ms = float(t.item())
    job_bytes = wl.job_bytes() if hasattr(wl, "job_bytes") else wl.bytes_per_step() * world
    value = job_bytes * K / (max_ms * 1e-3) / 1e9

    # ---- end to end through the C ABI with pinned host buffers (eager calls)
    e2e = None
    if not args.ncu:
        Ke = max(3, min(K, 200))
        ev2 = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in wl.groups]
               for _ in range(Ke)]
        def e2e_body(kv, s):
            # One decode step's worth of a group: the group's q (every layer)
            # from pinned host memory, its calls, its outputs back to pinned
            # host.  Both copies go through fr_copy_async (a kernel that
            # reaches the page-locked buffers through their device mapping).
            A.copy_async(wl.q, wl.q_host, stream=s)
            wl.run_group(A, kv, s)
            A.copy_async(wl.out_host, wl.out, stream=s)

        graphs_e2e = {}
        if use_graph:
            for kv in wl.groups:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    e2e_body(kv, torch.cuda.current_stream())
                graphs_e2e[kv] = g

        def e2e_group(kv):
            if use_graph:
                graphs_e2e[kv].replay()
            else:
                e2e_body(kv, stream)

        with torch.cuda.stream(stream):
            for kv in wl.groups:
                e2e_group(kv)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        with torch.cuda.stream(stream):
            for k in range(Ke):
                for i, kv in enumerate(wl.groups):
                    flush.fill_(i & 0xFF)
                    if align is not None:
                        dist.all_reduce(align)
                    ev2[k][i][0].record(stream)
                    e2e_group(kv)
                    ev2[k][i][1].record(stream)
        torch.cuda.synchronize()
        e_ms = sum(ev2[k][i][0].elapsed_time(ev2[k][i][1]) for k in range(Ke)
                   for i in range(len(wl.groups)))
        if world > 1:
            t = torch.tensor([e_ms], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        h2d, d2h = wl.e2e_bytes()
        e2e = {"value": job_bytes * Ke / (e_ms * 1e-3) / 1e9, "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "how": "per group of calls (one decode step's layers at one kv_len): one H2D of "
                      "every layer's q from pinned host, the calls through the C ABI, one D2H "
                      "of every output to pinned host, the copies by fr_copy_async (a kernel "
                      "reading/writing the page-locked buffers through their device mapping); "
                      "all three in one CUDA graph per group unless --no-graph; CUDA events "
                      "around them, L2 flushed before each group"}

    close = getattr(getattr(wl, "dec", None), "close", None)
    if close is not None:
        close()                          # collective: every rank frees its exchange buffer
    if rank != 0:
        return
    peak, peak_kind = peaks()
    sweep = {}
    for kv in wl.groups:
        us = group_ms[kv] * 1e3 / (K * wl.calls_per_group())
        gbs = wl.call_bytes(kv) / (us * 1e-6) / 1e9
        i = wl.groups.index(kv)
        per_step = np.array([ev[k][i][0].elapsed_time(ev[k][i][1]) for k in range(K)]) * 1e3 / \
            wl.calls_per_group()
        p10, p50, p90 = np.percentile(per_step, [10, 50, 90])
        sweep[str(kv)] = {"us_per_call": round(us, 3), "gbs": round(gbs, 1),
                          "frac_of_measured_hbm": round(gbs / peak, 4),
                          "us_per_call_p10_p50_p90": [round(float(p10), 3), round(float(p50), 3),
                                                      round(float(p90), 3)]}
    dom = str(wl.groups[-1])
    tr = traffic_per_launch() if args.workload == "cfg2" else None
    roofline = {
        "bound": "hbm",
        "kernel": f"split_decode_kernel (one fr_decode_attn call, merge fused), kv_len {dom}",
        "achieved": sweep[dom]["gbs"], "peak": peak, "unit": "GB/s",
        "frac": round(sweep[dom]["gbs"] / peak, 4), "peak_kind": peak_kind,
        "traffic": tr.get("dram_bytes_per_launch") if tr else None,
        "algorithmic_bytes_per_launch": wl.call_bytes(wl.groups[-1]),
    }
    cfg = wl.config()
    par = {"cfg2": f"dp{world} (one sequence per GPU)",
           "cfg3": f"{world} GPUs, (sequence, kv head) units by LPT, no collective",
           "cfg3p": f"{world} GPUs, sequences by LPT, no collective",
           "cfg4": f"{world} GPUs, KV range split, states exchanged ({args.exchange})"}[args.workload]
    cfg.update({"parallelism": par, "graph": use_graph,
                "launch_overlap": not args.no_overlap, "sweep": sweep})
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(max_ms / K, 5), "higher_is_better": True,
        "scaling": wl.scaling, "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
        "data": "synthetic N(0,1) fp16", "config": cfg, "roofline": roofline,
        "gpu_launches": int(launches_per_step * K), "e2e": e2e,
        "clocks": sampler.summary() if sampler else None,
    }
    if world == 1 and not args.no_cpu_baseline and not args.ncu and args.workload == "cfg2":
        line["cpu_baseline"] = cpu_baseline_cfg2(budget_s=12.0)
    emit(line)


# --------------------------------------------------------- reference arm
def _cfg2_host_problem(layers):
    """fp32 copies of cfg2 layers (K, V [16384, 2, 128]) and q per layer."""
    data = []
    for l in layers:
        k, v = W.cfg2_layer_kv(l)
        q = W.cfg2_layer_q(l)
        data.append((np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
                     np.ascontiguousarray(v, np.float32)))
    return data


class _RefRunner:
    """cpu_decode_attn calls over all host threads (oracle/_ref), else the C port."""

    def __init__(self, data, kv_lens):
        from oracle import oracle as O

        self.O = O
        self.lib = O.load_ref()
        self.kind = "reference" if self.lib is not None else "port"
        self.threads = os.cpu_count() or 1
        self.calls = [(q, k, v, kv) for kv in kv_lens for (q, k, v) in data]
        self.outs = [np.zeros((12, 128), np.float32) for _ in self.calls]
        f32p = ctypes.POINTER(ctypes.c_float)
        n = len(self.calls)
        if self.lib is not None:
            self.qs = (f32p * n)(*[q.ctypes.data_as(f32p) for q, _, _, _ in self.calls])
            self.ks = (f32p * n)(*[k.ctypes.data_as(f32p) for _, k, _, _ in self.calls])
            self.vs = (f32p * n)(*[v.ctypes.data_as(f32p) for _, _, v, _ in self.calls])
            self.os_ = (f32p * n)(*[o.ctypes.data_as(f32p) for o in self.outs])
            self.lens = (ctypes.c_int * n)(*[kv for _, _, _, kv in self.calls])

    def run(self):
        if self.lib is not None:
            self.lib.ref_cpu_decode_attn_many(self.qs, self.ks, self.vs, self.os_, self.lens,
                                              len(self.calls), 12, 2, 128, self.threads)
            return
        from concurrent.futures import ThreadPoolExecutor
        lib = self.O.load_oracle()
        f32p = ctypes.POINTER(ctypes.c_float)

        def one(i):
            q, k, v, kv = self.calls[i]
            lib.oracle_decode_attn_f32(q.ctypes.data_as(f32p), k.ctypes.data_as(f32p),
                                       v.ctypes.data_as(f32p), self.outs[i].ctypes.data_as(f32p),
                                       12, 2, 128, kv)

        with ThreadPoolExecutor(self.threads) as ex:
            list(ex.map(one, range(len(self.calls))))

    def bytes(self):
        return sum(W.decode_bytes([kv], 12, 2, 128) for _, _, _, kv in self.calls)


def cpu_baseline_cfg2(budget_s: float):
    """Bounded sample: 4 layers x the 4 kv_lens, repeated for about budget_s."""
    runner = _RefRunner(_cfg2_host_problem(range(4)), W.CFG2_KV_LENS)
    t0 = time.perf_counter()
    reps = 0
    while True:
        runner.run()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 2000:
            break
    return {"value": round(runner.bytes() * reps / el / 1e9, 4), "unit": UNIT,
            "cores": runner.threads, "kind": runner.kind,
            "sample": f"cfg2 layers 0-3 x kv_len {{512,2048,4096,16384}} (16 calls) x {reps} reps, "
                      f"{el:.1f} s; cpu_decode_attn (tests/test_kernels.cpp:229-270) on "
                      f"{runner.threads} threads"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    if args.workload != "cfg2":
        emit({"impl": "reference", "unavailable": f"reference arm implemented for cfg2 only"})
        return
    runner = _RefRunner(_cfg2_host_problem(range(W.CFG2_LAYERS)), W.CFG2_KV_LENS)
    for _ in range(args.warmup):
        runner.run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        runner.run()
    el = time.perf_counter() - t0
    value = runner.bytes() * args.steps / el / 1e9
    emit({
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32 (fp16-valued inputs)", "data": "synthetic N(0,1) fp16",
        "impl": "reference",
        "config": {"workload": "cfg2: Qwen2-1.5B-shape decode attention, batch 1 per GPU, 28 "
                               "layers x kv_len {512, 2048, 4096, 16384}",
                   "num_heads": 12, "num_kv_heads": 2, "head_dim": 128, "layers": 28,
                   "kv_lens": list(W.CFG2_KV_LENS)},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": runner.threads,
                         "kind": runner.kind,
                         "sample": "full cfg2 step (112 cpu_decode_attn calls) per step"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    })


def main():
    args = parse_args()
    rank, local_rank, world = dist_env()
    if args.gpus != world and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, torch, dist, rank, local_rank, world)
    finally:
        if world > 1:
            import gc
            gc.collect()                 # CUDA graphs holding NCCL work go first
            torch.cuda.synchronize()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
