#!/usr/bin/env python
"""Decode-attention benchmark (one JSON line on rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload cfg3|cfg2|cfg3p|cfg4|cfg1] [--layers L]

Headline (default, the same workload at every N): config 3, Qwen2-7B-shaped
batched decode attention - 64 sequences with ragged kv_len U{1024..8192}
(seed 2), H28 Hkv4 D128 - as one decode step of the model: its 28 layers'
attention calls back to back, each layer with its own KV pool, one batched
call (fr_decode_attn_batched) per layer, captured in one CUDA graph.  The
256 (sequence, kv head) units are split across the N GPUs
longest-processing-time first by token count, with no collective on the
data path; the total work is fixed ("strong").  value = the whole job's
algorithmic bytes (K+V of the valid range + q + out, every layer) / the
slowest rank's device time of the step.  A step's K/V (17 GB on one GPU,
2.1 GB per GPU at N=8) is far larger than L2, and L2 is also flushed (a
256 MiB write) before every step, outside the CUDA events.

Sub-records in the same line (sub.<name>), each with µs/call and GB/s:
  cfg3_call   one cold batched call of one layer per L2 flush (every N);
  cfg4        config 4, one 131072-position sequence (H28 Hkv4 D128) over 28
              layer caches; at N > 1 the KV range is split across the GPUs and
              the per-head (m, l, acc) states are exchanged inside the split
              kernel over NVLink (fr_decode_attn_exchange) (every N);
  cfg2        config 2, H12 Hkv2 D128, 28 layers x kv_len {512, 2048, 4096,
              16384}, with its own roofline (N = 1);
  cfg1        config 1, H14 Hkv2 D64 kv_len 512 over the 24 layers of a
              Qwen2-0.5B cache (N = 1).

--impl reference times the reference's own CPU implementation of the path
(cpu_decode_attn, tests/test_kernels.cpp:229-270, compiled from the
reference's sources into oracle/_ref; else the C port under oracle/) on the
headline workload's shapes with all host threads; rank 0 alone runs it.
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


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours",
                    help="reference = the reference's CPU implementation")
    ap.add_argument("--workload", choices=["cfg3", "cfg2", "cfg3p", "cfg4", "cfg1"],
                    default="cfg3")
    ap.add_argument("--layers", type=int, default=28,
                    help="cfg3/cfg4: layers decoded back to back per step")
    ap.add_argument("--page-size", type=int, default=16, help="cfg3p page rows (multiple of 16)")
    ap.add_argument("--page-order", choices=["shuffled", "sequential"], default="shuffled",
                    help="cfg3p: pages handed out in a seeded random order, or in order")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="cfg4 at N > 1: in-kernel peer exchange or NCCL all-gather")
    ap.add_argument("--no-graph", action="store_true", help="launch eagerly instead of graphs")
    ap.add_argument("--no-overlap", action="store_true",
                    help="disable launch overlap (pre-wait K/V prefetch under PDL)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="headline only, no sub-records")
    ap.add_argument("--shard", default=None, metavar="N:R",
                    help="development aid: time rank R's shard of an N-GPU run on this one GPU "
                         "(the line then describes that shard only)")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling run: headline only, no clocks/e2e/cpu legs")
    return ap.parse_args(argv)


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


def traffic_record(key: str):
    """DRAM bytes per launch of a kernel from a committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(key)
    except ValueError:
        return None


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


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


# --------------------------------------------------------------- workloads
# Each workload knows its shapes without a GPU (config(), used by both arms)
# and, once built on a device, runs one group of calls per key of `groups`.

def cfg3_config(world: int, layers: int) -> dict:
    lens = W.cfg3_lens()
    return {
        "workload": f"cfg3: Qwen2-7B-shape batched decode attention, 64 sequences, ragged kv_len "
                    f"U{{1024..8192}} (seed 2), {layers} layers per step, sharded by "
                    f"(sequence, kv head)",
        "shape": "Qwen2-7B attention (H28, Hkv4, D128), random data",
        "global_batch": 64, "num_heads": 28, "num_kv_heads": 4, "head_dim": 128,
        "layers": layers, "total_kv_tokens_per_layer": int(lens.sum()),
        "parallelism": f"{world} GPU(s), (sequence, kv head) units by LPT on token count, "
                       f"no collective",
        "l2": "step K/V far larger than L2; L2 also flushed (256 MiB write) before each step, "
              "outside the events",
    }


def cfg2_config(world: int) -> dict:
    return {
        "workload": "cfg2: Qwen2-1.5B-shape decode attention, batch 1 per GPU, 28 layers x "
                    "kv_len {512, 2048, 4096, 16384}",
        "shape": "Qwen2-1.5B attention (H12, Hkv2, D128), random data",
        "global_batch": world, "num_heads": 12, "num_kv_heads": 2, "head_dim": 128,
        "layers": 28, "kv_lens": list(W.CFG2_KV_LENS),
        "parallelism": f"{world} GPU(s), one sequence per GPU (weak)",
        "l2": "flushed (256 MiB write) before each kv_len group, outside the events",
    }


def cfg4_config(world: int, layers: int, exchange: str) -> dict:
    ex = "single GPU" if world == 1 else {
        "peer": "in-kernel peer stores over NVLink + merge (fr_decode_attn_exchange)",
        "nccl": "NCCL all-gather + merge kernel"}[exchange]
    return {
        "workload": f"cfg4: Qwen2-7B-shape long-context decode attention, 1 sequence, kv_len "
                    f"131072, {layers} layer(s) per step, KV range split across GPUs",
        "shape": "Qwen2-7B attention (H28, Hkv4, D128), random data",
        "global_batch": 1, "num_heads": 28, "num_kv_heads": 4, "head_dim": 128,
        "kv_len": 131072, "layers": layers, "exchange": ex,
        "parallelism": f"{world} GPU(s), contiguous KV ranges, (m, l, acc) states exchanged",
        "l2": "flushed (256 MiB write) before each step, outside the events; N > 1: ranks "
              "aligned by a one-element all-reduce after the flush",
    }


def cfg1_config(world: int) -> dict:
    return {
        "workload": "cfg1: Qwen2-0.5B-shape decode attention, kv_len 512, the 24 layers of one "
                    "decode step",
        "shape": "Qwen2-0.5B attention (H14, Hkv2, D64), random data",
        "global_batch": 1, "num_heads": 14, "num_kv_heads": 2, "head_dim": 64, "kv_len": 512,
        "layers": 24, "parallelism": "1 GPU",
        "l2": "flushed (256 MiB write) before each step, outside the events",
    }


class Cfg2:
    """28 layers x kv_len {512, 2048, 4096, 16384}, one sequence per rank."""

    L, S, H, HKV, D = W.CFG2_LAYERS, W.CFG2_MAX_SEQ, 12, 2, 128
    scaling = "weak"
    graphable = True
    align_ranks = False

    def __init__(self, torch, rank: int, world: int, device):
        g = torch.Generator(device=device)
        g.manual_seed(1 + 1000 * rank)
        self.world = world
        self.cache = torch.empty((self.L, 2, self.S, self.HKV, self.D), dtype=torch.float16,
                                 device=device)
        self.cache.normal_(generator=g)
        self.q = torch.empty((self.L, self.H, self.D), dtype=torch.float16, device=device)
        self.q.normal_(generator=g)
        self.out = torch.empty_like(self.q)
        self.groups = list(W.CFG2_KV_LENS)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()

    def call_bytes(self, kv) -> int:
        return W.decode_bytes([kv], self.H, self.HKV, self.D)

    def calls_per_group(self) -> int:
        return self.L

    def job_bytes_per_step(self) -> int:
        return sum(self.call_bytes(kv) * self.L for kv in self.groups) * self.world

    def workspace_bytes(self, A) -> int:
        return max(A.decode_workspace_size(1, self.H, self.HKV, self.D, kv) for kv in self.groups)

    def run_group(self, A, kv: int, stream) -> None:
        for l in range(self.L):
            A.decode_attn_v4_flash(self.q[l], self.cache[l, 0], self.cache[l, 1], self.out[l],
                                   self.H, self.HKV, self.D, kv, stream)

    def e2e_bytes(self):
        per = self.L * self.H * self.D * 2 * len(self.groups)
        return per, per

    def config(self):
        return cfg2_config(self.world)


class Cfg1(Cfg2):
    """Config 1's shape over the 24 layers of a Qwen2-0.5B cache at kv_len 512."""

    L, S, H, HKV, D = 24, 512, 14, 2, 64

    def __init__(self, torch, rank: int, world: int, device):
        g = torch.Generator(device=device)
        g.manual_seed(0)
        self.world = world
        self.cache = torch.empty((self.L, 2, self.S, self.HKV, self.D), dtype=torch.float16,
                                 device=device).normal_(generator=g)
        self.q = torch.empty((self.L, self.H, self.D), dtype=torch.float16,
                             device=device).normal_(generator=g)
        self.out = torch.empty_like(self.q)
        self.groups = [512]

    def config(self):
        return cfg1_config(self.world)


class Cfg3:
    """Qwen2-7B batched decode: 64 sequences, kv_len ~ U{1024..8192} (seed 2),
    H28 Hkv4 D128, `layers` layers per step.  The 256 (sequence, kv head)
    units are assigned to ranks by LPT on token count; each rank keeps its
    units in one KV pool per layer [rows, 1, 128] (a unit is one kv head with
    its 7 query heads) and makes one batched call per layer."""

    H, HKV, D, G = 28, 4, 128, 7
    scaling = "strong"
    graphable = True
    align_ranks = False

    def __init__(self, torch, rank: int, world: int, device, layers: int = 1):
        from forgert_b200 import sharding as SH
        self.world = world
        self.L = max(1, layers)
        self.lens_all = W.cfg3_lens()
        mine = SH.shard_batched(self.lens_all, self.HKV, world)[rank]
        lens = [u[2] for u in mine]
        self.U = len(mine)
        rows = int(sum(lens))
        offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        g = torch.Generator(device=device)
        g.manual_seed(2 + 1000 * rank)
        shp = (self.L, rows, 1, self.D)
        self.kpool = torch.empty(shp, dtype=torch.float16, device=device).normal_(generator=g)
        self.vpool = torch.empty(shp, dtype=torch.float16, device=device).normal_(generator=g)
        self.offs = torch.from_numpy(offs).to(device)
        self.lens = torch.tensor(lens, dtype=torch.int32, device=device)
        self.q = torch.empty((self.L, self.U, self.G, self.D), dtype=torch.float16,
                             device=device).normal_(generator=g)
        self.out = torch.empty_like(self.q)
        self.rows = rows
        self.max_len = int(max(lens))
        self.groups = ["step"]
        self.my_call_bytes = W.decode_bytes(lens, self.G, 1, self.D)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()

    def call_bytes(self, key=None) -> int:
        return self.my_call_bytes

    def calls_per_group(self) -> int:
        return self.L

    def job_bytes_per_step(self) -> int:
        return W.decode_bytes(self.lens_all, self.H, self.HKV, self.D) * self.L

    def workspace_bytes(self, A) -> int:
        return A.decode_workspace_size(self.U, self.G, 1, self.D, self.max_len)

    def run_group(self, A, key, stream) -> None:
        for l in range(self.L):
            self.run_layer(A, key, l, stream)

    def run_layer(self, A, key, l: int, stream) -> None:
        A.decode_attn_batched(self.q[l], self.kpool[l], self.vpool[l], self.offs, self.lens,
                              self.out[l], self.U, self.G, 1, self.D, self.rows, self.max_len,
                              stream)

    def e2e_bytes(self):
        n = self.L * self.U * self.G * self.D * 2
        return n, n

    def config(self):
        return cfg3_config(self.world, self.L)


class Cfg3Paged(Cfg3):
    """cfg3's 64 sequences in a paged KV cache: pages of page_size rows x 4 kv heads
    x 128, handed out in a seeded random order (a fragmented serving cache),
    one block table per sequence, one fr_decode_attn_paged call (one layer).
    N GPUs: whole sequences are assigned by LPT on length; no collective."""

    def __init__(self, torch, rank: int, world: int, device, page_size: int = 16,
                 page_order: str = "shuffled"):
        from forgert_b200 import sharding as SH
        self.world = world
        self.L = 1
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
        self.q = torch.empty((self.B, self.H, self.D), dtype=torch.float16,
                             device=device).normal_(generator=g)
        self.out = torch.empty_like(self.q)
        self.max_len = int(max(lens))
        self.groups = ["step"]
        self.my_call_bytes = W.decode_bytes(lens, self.H, self.HKV, self.D)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()
        self.U = self.B

    def workspace_bytes(self, A) -> int:
        return A.decode_workspace_size(self.B, self.H, self.HKV, self.D, self.max_len)

    run_layer = None        # one call per step: the serial end-to-end form

    def run_group(self, A, key, stream) -> None:
        A.decode_attn_paged(self.q, self.kpages, self.vpages, self.table, self.lens, self.out,
                            self.B, self.H, self.HKV, self.D, self.PAGE, self.num_pages,
                            self.width, self.max_len, stream)

    def e2e_bytes(self):
        n = self.B * self.H * self.D * 2
        return n, n

    def config(self):
        c = cfg3_config(self.world, 1)
        c["workload"] = (f"cfg3p: cfg3's 64 sequences in a paged KV cache ({self.PAGE}-row pages "
                         f"in {self.page_order} order, block table per sequence), one layer, "
                         f"sharded by sequence")
        c["page_size"] = self.PAGE
        return c


class Cfg4:
    """Qwen2-7B long context: one sequence, kv_len 131072, H28 Hkv4 D128,
    `layers` layer caches per step.  One GPU: plain fr_decode_attn calls.
    N GPUs: each rank holds a contiguous KV range; exchange "peer": one
    fr_decode_attn_exchange kernel per rank and layer computes its states,
    stores them into every rank's exchange buffer over NVLink and merges what
    arrives; "nccl": partial kernel, NCCL all-gather of the states, merge
    kernel.  Total work is fixed ("strong")."""

    H, HKV, D, T = 28, 4, 128, 131072
    scaling = "strong"
    graphable = True

    def __init__(self, torch, rank: int, world: int, device, exchange: str = "peer",
                 layers: int = 1, shard: tuple[int, int] | None = None):
        from forgert_b200 import sharding as SH
        self.world = world
        self.L = max(1, layers)
        n_split, r_split = shard if shard else (world, rank)
        b, e = SH.kv_ranges(self.T, n_split)[r_split]
        self.n = e - b
        g = torch.Generator(device=device)
        g.manual_seed(3 + 1000 * r_split)
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
        self.my_call_bytes = W.decode_bytes([self.n], self.H, self.HKV, self.D)
        self.q_host = self.q.cpu().pin_memory()
        self.out_host = torch.empty_like(self.q_host).pin_memory()
        self.n_split = n_split

    def call_bytes(self, key=None) -> int:
        return self.my_call_bytes

    def calls_per_group(self) -> int:
        return self.L

    def job_bytes_per_step(self) -> int:
        return W.decode_bytes([self.T], self.H, self.HKV, self.D) * self.L

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
        return cfg4_config(self.world, self.L, self.exchange if self.world > 1 else "peer")

    def close(self):
        if self.dec is not None and hasattr(self.dec, "close"):
            self.dec.close()       # collective: every rank frees its exchange buffer


# ------------------------------------------------------------- timing core
class Timer:
    """Warm-up, CUDA-graph capture and event timing of one workload."""

    def __init__(self, ctx, wl, use_graph: bool):
        self.ctx, self.wl = ctx, wl
        torch, A, lib, stream = ctx.torch, ctx.A, ctx.lib, ctx.stream
        A.reserve_workspace(wl.workspace_bytes(A))
        torch.cuda.synchronize()
        # eager warm-up (creates the library's device state outside capture)
        with torch.cuda.stream(stream):
            for key in wl.groups:
                wl.run_group(A, key, stream)
        torch.cuda.synchronize()
        self.use_graph = use_graph and wl.graphable
        self.graphs = {}
        self.launches_per_step = 0
        if self.use_graph:
            for key in wl.groups:
                g = torch.cuda.CUDAGraph()
                c0 = lib.fr_launch_count()
                with torch.cuda.graph(g, stream=stream):
                    wl.run_group(A, key, torch.cuda.current_stream())
                self.launches_per_step += lib.fr_launch_count() - c0
                self.graphs[key] = g
        else:
            c0 = lib.fr_launch_count()
            with torch.cuda.stream(stream):
                for key in wl.groups:
                    wl.run_group(A, key, stream)
            torch.cuda.synchronize()
            self.launches_per_step = lib.fr_launch_count() - c0
        self.align = (torch.zeros(1, dtype=torch.float32, device=ctx.device)
                      if ctx.world > 1 and getattr(wl, "align_ranks", False) else None)

    def _group(self, key, body=None):
        if body is not None:
            body(key)
        elif self.use_graph:
            self.graphs[key].replay()
        else:
            self.wl.run_group(self.ctx.A, key, self.ctx.stream)

    def run(self, steps: int, warmup: int, body=None, sampler=None):
        """Times `steps` steps after `warmup` untimed ones; every group of a
        step is bracketed by its own events after an L2 flush (and, for
        workloads whose ranks wait for each other, a rank alignment).
        Returns (per-group total ms, per-group per-step ms arrays, max-over-
        ranks total ms)."""
        ctx, wl = self.ctx, self.wl
        torch, dist, stream = ctx.torch, ctx.dist, ctx.stream

        def step(events):
            for i, key in enumerate(wl.groups):
                ctx.flush.fill_(i & 0xFF)
                if self.align is not None:
                    dist.all_reduce(self.align)
                if events is not None:
                    events[i][0].record(stream)
                self._group(key, body)
                if events is not None:
                    events[i][1].record(stream)

        with torch.cuda.stream(stream):
            for _ in range(warmup):
                step(None)
        torch.cuda.synchronize()
        if ctx.world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in wl.groups]
              for _ in range(steps)]
        if sampler:
            sampler.__enter__()
        with torch.cuda.stream(stream):
            for k in range(steps):
                step(ev[k])
        torch.cuda.synchronize()
        if sampler:
            sampler.__exit__()
        if ctx.world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        per = {key: np.array([ev[k][i][0].elapsed_time(ev[k][i][1]) for k in range(steps)])
               for i, key in enumerate(wl.groups)}
        tot = {key: float(v.sum()) for key, v in per.items()}
        total = sum(tot.values())
        mx = total
        if ctx.world > 1:
            t = torch.tensor([total], dtype=torch.float64, device=ctx.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            mx = float(t.item())
        assert ctx.A.device_error() == 0, "in-kernel wait timed out"
        return tot, per, mx

    def release(self):
        self.graphs.clear()


class Ctx:
    def __init__(self, torch, dist, A, lib, device, stream, flush, rank, world):
        self.torch, self.dist, self.A, self.lib = torch, dist, A, lib
        self.device, self.stream, self.flush = device, stream, flush
        self.rank, self.world = rank, world


def group_stats(wl, tot, per, steps, peak):
    out = {}
    for key in wl.groups:
        us = tot[key] * 1e3 / (steps * wl.calls_per_group())
        gbs = wl.call_bytes(key) / (us * 1e-6) / 1e9
        p10, p50, p90 = np.percentile(per[key] * 1e3 / wl.calls_per_group(), [10, 50, 90])
        out[str(key)] = {"us_per_call": round(us, 3), "gbs_per_gpu": round(gbs, 1),
                         "frac_of_measured_hbm": round(gbs / peak, 4),
                         "us_per_call_p10_p50_p90": [round(float(p10), 3), round(float(p50), 3),
                                                     round(float(p90), 3)]}
    return out


def run_sub(ctx, name, make, steps, warmup, use_graph, peak):
    """One sub-record: build, time, summarise, free."""
    torch = ctx.torch
    wl = make()
    tm = Timer(ctx, wl, use_graph)
    tot, per, mx = tm.run(steps, warmup)
    rec = {"config": wl.config(), "steps": steps, "warmup": warmup,
           "ms_per_step": round(mx / steps, 5),
           "value": round(wl.job_bytes_per_step() * steps / (mx * 1e-3) / 1e9, 2),
           "unit": UNIT, "scaling": wl.scaling,
           "per_call": group_stats(wl, tot, per, steps, peak),
           "gpu_launches_per_step": int(tm.launches_per_step)}
    tm.release()
    if hasattr(wl, "close"):
        wl.close()
    del wl, tm
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return rec


def run_ours(args, torch, dist, rank, local_rank, world):
    from forgert_b200 import _lib
    from forgert_b200 import attention as A

    lib = _lib.load()
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    shard = None
    if args.shard:
        n, r = (int(x) for x in args.shard.split(":"))
        shard = (n, r)
    wrank, wworld = shard[1] if shard else rank, shard[0] if shard else world

    def make(workload, layers):
        if workload == "cfg2":
            return Cfg2(torch, wrank, wworld, device)
        if workload == "cfg1":
            return Cfg1(torch, wrank, wworld, device)
        if workload == "cfg3":
            return Cfg3(torch, wrank, wworld, device, layers)
        if workload == "cfg3p":
            return Cfg3Paged(torch, wrank, wworld, device, args.page_size, args.page_order)
        return Cfg4(torch, rank, world, device, args.exchange, layers, shard=shard)

    stream = torch.cuda.Stream(device)
    # Decode-step launch overlap: the attention kernel may stream K/V rows
    # older than the newest one while the preceding kernel finishes.
    lib.fr_set_launch_overlap(0 if args.no_overlap else 1)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    ctx = Ctx(torch, dist, A, lib, device, stream, flush, rank, world)
    peak, peak_kind = peaks()
    use_graph = not args.no_graph

    # ------------------------------------------------------------ headline
    wl = make(args.workload, args.layers)
    tm = Timer(ctx, wl, use_graph)
    sampler = ClockSampler(local_rank) if not args.ncu else None
    tot, per, max_ms = tm.run(args.steps, args.warmup, sampler=sampler)
    K = args.steps
    job_bytes = wl.job_bytes_per_step()
    if shard:
        job_bytes = wl.call_bytes(wl.groups[0]) * wl.calls_per_group() * len(wl.groups)
    value = job_bytes * K / (max_ms * 1e-3) / 1e9
    stats = group_stats(wl, tot, per, K, peak)

    # ---- end to end through the C ABI with pinned host buffers
    e2e = None
    if not args.ncu and hasattr(wl, "q_host"):
        side = torch.cuda.Stream(device)
        layered = getattr(wl, "run_layer", None) is not None

        def e2e_body(key, s=None):
            # One decode step's worth of a group: its q (every layer) from
            # pinned host memory, its calls, its outputs back to pinned host.
            # One call per step: both copies through fr_copy_async (a kernel
            # that reaches the page-locked buffers through their device
            # mapping).  Per-layer workloads overlap them with the calls on a
            # side stream, by the copy engines (no SM time taken from the
            # calls): the q of the first ceil(L/8) layers in one copy the
            # first call waits for, the other layers' q in a second copy
            # (done long before its first layer starts) - every wait between
            # two calls costs their launch overlap, so there is one; each
            # layer's output leaves while later layers compute, and the step
            # ends when the last output has landed.
            s = s or stream
            if not layered:
                A.copy_async(wl.q, wl.q_host, stream=s)
                wl.run_group(A, key, s)
                A.copy_async(wl.out_host, wl.out, stream=s)
                return
            side.wait_stream(s)
            k = -(-wl.L // 8)
            ready = [torch.cuda.Event(), torch.cuda.Event()]
            done = [torch.cuda.Event() for _ in range(wl.L)]
            with torch.cuda.stream(side):
                wl.q[:k].copy_(wl.q_host[:k], non_blocking=True)
                ready[0].record(side)
                if k < wl.L:
                    wl.q[k:].copy_(wl.q_host[k:], non_blocking=True)
                    ready[1].record(side)
            for l in range(wl.L):
                if l == 0 or l == k:
                    s.wait_event(ready[0 if l == 0 else 1])
                wl.run_layer(A, key, l, s)
                done[l].record(s)
                side.wait_event(done[l])
                with torch.cuda.stream(side):
                    wl.out_host[l].copy_(wl.out[l], non_blocking=True)
            s.wait_stream(side)

        graphs_e2e = {}
        if tm.use_graph:
            for key in wl.groups:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    e2e_body(key, torch.cuda.current_stream())
                graphs_e2e[key] = g
        body = (lambda key: graphs_e2e[key].replay()) if tm.use_graph else e2e_body
        Ke = max(3, min(K, 200))
        _, _, e_ms = tm.run(Ke, 2, body=body)
        h2d, d2h = wl.e2e_bytes()
        e2e = {"value": round(job_bytes * Ke / (e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "how": ("per step: every layer's q from pinned host memory, the calls through "
                       "the C ABI, every output to pinned host memory; " +
                       ("the copies by the copy engines on a second stream, overlapping the "
                        "calls (q of the first ceil(L/8) layers before the first call, the "
                        "rest in one copy the call of layer ceil(L/8) waits for; each output "
                        "as soon as its layer is done); " if layered else
                        "one copy each way around the calls by fr_copy_async (a kernel "
                        "that reads/writes the page-locked buffers through their device "
                        "mapping); ") +
                       "all in one CUDA graph per step; CUDA events around them, L2 flushed "
                       "before each step")}
        graphs_e2e.clear()
    tm.release()
    launches = int(tm.launches_per_step * K)
    if hasattr(wl, "close"):
        wl.close()
    dom_key = wl.groups[-1]
    head_calls = wl.calls_per_group()
    head_call_bytes = wl.call_bytes(dom_key)
    cfg = wl.config()
    del wl, tm
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    # ------------------------------------------------------- sub-records
    sub = {}
    if not args.ncu and not args.no_sub and not shard and args.workload == "cfg3":
        Ks = max(5, min(K, 50))
        sub["cfg3_call"] = run_sub(ctx, "cfg3_call", lambda: Cfg3(torch, rank, world, device, 1),
                                   max(20, min(K, 200)), 5, use_graph, peak)
        sub["cfg4"] = run_sub(ctx, "cfg4",
                              lambda: Cfg4(torch, rank, world, device, args.exchange, 28),
                              Ks, 3, use_graph, peak)
        if world == 1:
            sub["cfg2"] = run_sub(ctx, "cfg2", lambda: Cfg2(torch, 0, 1, device), Ks * 4, 5,
                                  use_graph, peak)
            c2 = sub["cfg2"]["per_call"]["16384"]
            tr = traffic_record("cfg2_kv16384")
            sub["cfg2"]["roofline"] = {
                "bound": "hbm", "kernel": "split_decode_kernel (one fr_decode_attn call, merge "
                                          "fused), kv_len 16384",
                "achieved": c2["gbs_per_gpu"], "peak": peak, "unit": "GB/s",
                "frac": round(c2["gbs_per_gpu"] / peak, 4), "peak_kind": peak_kind,
                "traffic": tr.get("dram_bytes_per_launch") if tr else None,
                "algorithmic_bytes_per_launch": W.decode_bytes([16384], 12, 2, 128)}
            sub["cfg1"] = run_sub(ctx, "cfg1", lambda: Cfg1(torch, 0, 1, device), Ks * 4, 5,
                                  use_graph, peak)
    if rank != 0:
        return

    tr = traffic_record(f"{args.workload}_call") if args.workload in ("cfg3", "cfg4") else \
        traffic_record("cfg2_kv16384") if args.workload == "cfg2" else None
    achieved = head_call_bytes / (stats[str(dom_key)]["us_per_call"] * 1e-6) / 1e9
    kern = {"cfg3": "persistent_decode_kernel (fr_decode_attn_batched): one call per layer",
            "cfg3p": "split_decode_kernel, paged (fr_decode_attn_paged)",
            "cfg4": "split_decode_kernel (fr_decode_attn / fr_decode_attn_exchange), one call "
                    "per layer",
            "cfg2": "split_decode_kernel (fr_decode_attn), kv_len 16384",
            "cfg1": "split_decode_kernel (fr_decode_attn), kv_len 512"}[args.workload]
    roofline = {
        "bound": "hbm", "kernel": kern, "achieved": round(achieved, 1), "peak": peak,
        "unit": "GB/s", "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
        # DRAM bytes of one full-size capture, scaled to this GPU's call by
        # the algorithmic bytes it processes (traffic grows with them)
        "traffic": (int(tr["dram_bytes_per_launch"] * head_call_bytes /
                        tr["algorithmic_bytes_per_launch"]) if tr else None),
        "traffic_scope": (f"{tr.get('scope')}, scaled to this call's algorithmic bytes"
                          if tr else None),
        "algorithmic_bytes_per_launch": head_call_bytes,
        "how": "achieved = algorithmic bytes of one call on this GPU / (device time of the "
               "timed steps / calls per step); rank 0's calls",
    }
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(max_ms / K, 5), "higher_is_better": True,
        "scaling": "strong" if args.workload in ("cfg3", "cfg4", "cfg3p") else "weak",
        "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)",
        "data": "synthetic N(0,1) fp16", "config": cfg,
        "per_call": stats, "calls_per_step": head_calls,
        "method": {"graph": use_graph, "launch_overlap": not args.no_overlap},
        "roofline": roofline, "gpu_launches": launches, "e2e": e2e,
        "clocks": sampler.summary() if sampler else None,
    }
    if shard:
        line["shard"] = {"of_gpus": shard[0], "rank": shard[1],
                         "note": "one rank's shard timed alone on one GPU; value = this shard's "
                                 "bytes / its time, not a whole-job figure"}
    if sub:
        line["sub"] = sub
    if world == 1 and not shard and not args.no_cpu_baseline and not args.ncu and \
            args.workload == "cfg3":
        # in a fresh process, as the reference arm runs: none of this
        # process's threads, pinned buffers or allocator state competes
        import multiprocessing as mp
        with mp.get_context("spawn").Pool(1) as pool:
            line["cpu_baseline"] = pool.apply(cpu_baseline_cfg3, (12.0,))
            line["cpu_baseline_hf"] = pool.apply(cpu_baseline_hf_cfg3, (8.0,))
    emit(line)


# --------------------------------------------------------- reference arm
class _RefRunner:
    """cpu_decode_attn (the reference's own CPU path, oracle/_ref; else the C
    port) over a list of calls, one host thread per core pulling calls off a
    queue longest first, so no thread idles while long calls remain."""

    def __init__(self, calls, H, Hkv, D):
        from oracle import oracle as O

        self.lib = O.load_ref()
        self.kind = "reference" if self.lib is not None else "port"
        self.fn = (self.lib.ref_cpu_decode_attn if self.lib is not None
                   else O.load_oracle().oracle_decode_attn_f32)
        self.threads = os.cpu_count() or 1
        self.H, self.Hkv, self.D = H, Hkv, D
        self.calls = sorted(calls, key=lambda c: -c[3])     # (q, k, v, kv_len)
        self.outs = [np.zeros((H, D), np.float32) for _ in self.calls]

    def run(self, calls=None):
        import queue
        f32p = ctypes.POINTER(ctypes.c_float)
        idx = range(len(self.calls)) if calls is None else calls
        qu = queue.SimpleQueue()
        for i in idx:
            qu.put(i)

        def worker():
            while True:
                try:
                    i = qu.get_nowait()
                except queue.Empty:
                    return
                q, k, v, n = self.calls[i]
                self.fn(q.ctypes.data_as(f32p), k.ctypes.data_as(f32p), v.ctypes.data_as(f32p),
                        self.outs[i].ctypes.data_as(f32p), self.H, self.Hkv, self.D, n)

        ts = [threading.Thread(target=worker) for _ in range(self.threads)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    def bytes(self, calls=None):
        idx = range(len(self.calls)) if calls is None else calls
        return sum(W.decode_bytes([self.calls[i][3]], self.H, self.Hkv, self.D) for i in idx)


def _cfg3_host_calls(max_seqs=None):
    """fp32 host copies of cfg3's sequences (q [28,128], K/V [len,4,128])."""
    lens, q, ks, vs = W.cfg3_inputs(max_seqs=max_seqs)
    return [(np.ascontiguousarray(q[b], np.float32), np.ascontiguousarray(ks[b], np.float32),
             np.ascontiguousarray(vs[b], np.float32), int(lens[b])) for b in range(len(ks))]


def _sample_for(runner, budget_s, min_frac=0.25):
    """Calls of a bounded sample: every call (one layer of the batch) when one
    pass fits the budget, else the longest-first prefix that does, at least
    `min_frac` of the calls, interleaved long and short."""
    t0 = time.perf_counter()
    runner.run()
    one = time.perf_counter() - t0
    n = len(runner.calls)
    if one <= budget_s:
        return list(range(n)), one
    k = max(int(n * min_frac), int(n * budget_s / one))
    order = [i for pair in zip(range(n), range(n - 1, -1, -1)) for i in pair]
    seen, out = set(), []
    for i in order:
        if i not in seen:
            seen.add(i)
            out.append(i)
        if len(out) >= k:
            break
    return out, one


def cpu_baseline_cfg3(budget_s: float):
    """The reference's cpu_decode_attn over one layer of cfg3's 64 sequences,
    repeated for about budget_s on all host threads."""
    runner = _RefRunner(_cfg3_host_calls(), 28, 4, 128)
    runner.run()                                   # warm (page in the inputs)
    t0 = time.perf_counter()
    reps = 0
    while True:
        runner.run()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    return {"value": round(runner.bytes() * reps / el / 1e9, 4), "unit": UNIT,
            "cores": runner.threads, "cpu": cpu_model(), "kind": runner.kind,
            "sample": f"one layer of cfg3 (64 sequences, H28 Hkv4 D128, ragged kv_len) x {reps} "
                      f"reps, {el:.1f} s; cpu_decode_attn (tests/test_kernels.cpp:229-270) per "
                      f"sequence on {runner.threads} threads, longest sequences first from a "
                      f"shared queue; fp32 inputs as that function takes them"}


def cpu_baseline_hf_cfg3(budget_s: float):
    """transformers' eager attention (python/reference.py's arithmetic:
    Qwen2 eager_attention_forward, fp16 on CPU, probabilities rounded to fp16)
    on cfg3 sequences, torch threads = all host cores."""
    try:
        import torch
        from transformers.models.qwen2.modeling_qwen2 import eager_attention_forward
    except Exception as e:        # pragma: no cover - transformers is in the image
        return {"unavailable": f"transformers not importable: {e}"}
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    class _Mod(torch.nn.Module):
        num_key_value_groups = 7

    mod = _Mod().eval()
    lens, q, ks, vs = W.cfg3_inputs(max_seqs=16)
    tq = [torch.from_numpy(q[b]).view(1, 28, 1, 128) for b in range(len(ks))]
    tk = [torch.from_numpy(np.ascontiguousarray(k.transpose(1, 0, 2)))[None] for k in ks]
    tv = [torch.from_numpy(np.ascontiguousarray(v.transpose(1, 0, 2)))[None] for v in vs]
    scaling = 128 ** -0.5
    with torch.no_grad():
        eager_attention_forward(mod, tq[0], tk[0], tv[0], None, scaling)
        t0 = time.perf_counter()
        done = 0
        nbytes = 0
        while True:
            for b in range(len(ks)):
                eager_attention_forward(mod, tq[b], tk[b], tv[b], None, scaling)
                nbytes += W.decode_bytes([int(lens[b])], 28, 4, 128)
            done += 1
            el = time.perf_counter() - t0
            if el >= budget_s or done >= 1000:
                break
    return {"value": round(nbytes / el / 1e9, 4), "unit": UNIT, "cores": threads,
            "cpu": cpu_model(), "kind": "reference",
            "sample": f"cfg3 sequences 0-15 (H28 Hkv4 D128) x {done} reps, {el:.1f} s; "
                      f"transformers Qwen2 eager_attention_forward (python/reference.py's "
                      f"attention), fp16 CPU tensors, torch.set_num_threads({threads})"}


def run_reference(args, rank, world):
    """The reference's CPU path on the headline workload's shapes (cfg3): one
    step = one layer of the 64-sequence batch (or, when K+W such steps would
    exceed about a minute, a bounded longest-and-shortest sample of it)."""
    if rank != 0:
        return
    if args.workload != "cfg3":
        emit({"impl": "reference", "unavailable": "reference arm implemented for the default "
                                                  "workload (cfg3) only"})
        return
    runner = _RefRunner(_cfg3_host_calls(), 28, 4, 128)
    budget = 60.0 / max(1, args.steps + args.warmup)
    calls, one = _sample_for(runner, budget)
    for _ in range(args.warmup):
        runner.run(calls)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        runner.run(calls)
    el = time.perf_counter() - t0
    value = runner.bytes(calls) * args.steps / el / 1e9
    sample = (f"{len(calls)} of cfg3's 64 sequences (one layer, H28 Hkv4 D128) per step; "
              f"cpu_decode_attn (tests/test_kernels.cpp:229-270) per sequence on "
              f"{runner.threads} threads, longest first from a shared queue")
    emit({
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32 (fp16-valued inputs)", "data": "synthetic N(0,1) fp16",
        "impl": "reference", "config": cfg3_config(world, args.layers),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": runner.threads,
                         "cpu": cpu_model(), "kind": runner.kind, "sample": sample},
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
