"""Per-phase timeline of the decode kernels inside a decode step (diagnostics).

  python -m forgert_b200.phase_trace --workload cfg2 --kv 16384 [--no-overlap] [--gemm]
  python -m forgert_b200.phase_trace --workload cfg3 --shard 8:0

Runs the trace build of the library (libforgert_b200_trace.so, built here
with `python -m forgert_b200.build --trace`): every CTA of the split kernel
(fr_decode_attn) and of the persistent batched kernel (fr_decode_attn_batched)
appends %globaltimer stamps at its phase boundaries (forgert_b200/csrc/
trace.cuh).  The workload is a decode step's chain of layer calls captured
in one CUDA graph, as bench.py times it:

  cfg2  H12 Hkv2 D128, 28 layers of a [28, 2, 16384, 2, 128] cache at one kv_len;
  cfg3  Qwen2-7B batched (64 ragged sequences, H28 Hkv4 D128), rank R's
        (sequence, kv head) units of an N-GPU split, 28 layer pools.

--no-overlap turns launch overlap off (no K/V prefetch before the
dependency wait); --gemm puts a 4096^3 fp16 GEMM (torch) between the layer
calls, as the reference's executor runs projections between attention calls.

Prints one JSON object: per phase, the median over the traced launches of
the median and the latest CTA, in microseconds from the launch's first CTA
start, plus the launch-to-launch period.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
EVENTS = {1: "start", 2: "meta", 3: "first_issue", 4: "dep_wait", 5: "q_loaded",
          6: "first_full", 7: "loop_end", 8: "fold", 9: "stored", 10: "merge_end",
          11: "xmerge_end", 12: "end", 13: "counted", 14: "merge_begin",
          15: "merge_loaded", 16: "fold_synced", 17: "state_done", 18: "cluster_ready",
          19: "recv_done", 20: "fold_stored", 21: "fold_weights"}


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=["cfg2", "cfg3"], default="cfg2")
    ap.add_argument("--kv", type=int, default=16384, help="cfg2 kv_len")
    ap.add_argument("--shard", default="1:0", help="cfg3: N:R, rank R's units of an N-GPU split")
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--replays", type=int, default=4)
    ap.add_argument("--no-overlap", action="store_true")
    ap.add_argument("--gemm", action="store_true")
    ap.add_argument("--dump", default=None, help="also save the raw records (.npz, one array per CTA)")
    ap.add_argument("--lib", default=None,
                    help="trace build to load (default: libforgert_b200_trace.so, built if missing)")
    return ap.parse_args(argv)


def load_trace_lib(path=None):
    from . import build as B
    path = Path(path) if path else B.TRACE_LIB_PATH
    if not path.exists():
        B.build(trace=True)
    os.environ["FORGERT_B200_LIB"] = str(path)
    from . import _lib
    lib = _lib.load()
    lib.fr_trace_attach.restype = ctypes.c_int
    lib.fr_trace_attach.argtypes = [ctypes.c_void_p]
    return lib


MAX_CTAS, PER_CTA = 2048, 128 * 32      # kTraceMaxCtas, kTraceLaunches x kTraceEvents (csrc/trace.cuh)
# launch = low 32 bits of the grid's %gridid (one value per launch)
REC = np.dtype([("t", "<u8"), ("launch", "<u4"), ("ev_sm", "<u4")])


def records_by_cta(raw: np.ndarray) -> dict:
    """raw: the attached buffer as [MAX_CTAS, PER_CTA] records.  Returns
    {cta: its non-empty records in time order}."""
    out = {}
    for c in range(raw.shape[0]):
        r = raw[c][raw[c]["t"] != 0]
        if r.size:
            out[c] = np.sort(r, order="t")
    return out


def build_cfg2(torch, args, A, dev):
    L, H, Hkv, D = args.layers, 12, 2, 128
    g = torch.Generator(device=dev).manual_seed(1)
    cache = torch.empty((L, 2, 16384, Hkv, D), dtype=torch.float16, device=dev).normal_(generator=g)
    q = torch.empty((L, H, D), dtype=torch.float16, device=dev).normal_(generator=g)
    out = torch.empty_like(q)
    A.reserve_workspace(A.decode_workspace_size(1, H, Hkv, D, args.kv))

    def call(l, s):
        A.decode_attn_v4_flash(q[l], cache[l, 0], cache[l, 1], out[l], H, Hkv, D, args.kv, s)
    return call


def build_cfg3(torch, args, A, dev):
    from . import sharding as SH
    from . import workloads as W
    n, r = (int(x) for x in args.shard.split(":"))
    lens = [u[2] for u in SH.shard_batched(W.cfg3_lens(), 4, n)[r]]
    U, rows, L, G, D = len(lens), int(sum(lens)), args.layers, 7, 128
    offs = torch.tensor(np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64), device=dev)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(2)
    kp = torch.empty((L, rows, 1, D), dtype=torch.float16, device=dev).normal_(generator=g)
    vp = torch.empty_like(kp).normal_(generator=g)
    q = torch.empty((L, U, G, D), dtype=torch.float16, device=dev).normal_(generator=g)
    out = torch.empty_like(q)
    A.reserve_workspace(A.decode_workspace_size(U, G, 1, D, max(lens)))

    def call(l, s):
        A.decode_attn_batched(q[l], kp[l], vp[l], offs, lens_d, out[l], U, G, 1, D, rows,
                              max(lens), s)
    return call


def summarise(per_cta):
    """per_cta: {cta: records (t, launch, ev_sm)}.  For each launch,
    phases are timed from the launch's earliest CTA start; reported as the
    median over launches of the median CTA (first occurrence of the event in
    the CTA), of the median CTA's last occurrence (per-item events of the
    persistent kernel: the end of its range) and of the latest CTA (last
    occurrence)."""
    launches: dict[int, dict[str, dict[int, list]]] = {}
    for cta, recs in per_cta.items():
        for t, k, evsm in zip(recs["t"], recs["launch"], recs["ev_sm"]):
            name = EVENTS.get(int(evsm) & 0xFF, str(int(evsm) & 0xFF))
            launches.setdefault(int(k), {}).setdefault(name, {}).setdefault(cta, []).append(int(t))
    ks = sorted(k for k, d in launches.items() if "start" in d)
    ks = ks[1:-1] if len(ks) > 2 else ks          # drop the edges of the traced window
    starts, phases = [], {}
    for k in ks:
        d = launches[k]
        t0 = min(min(v) for v in d["start"].values())
        starts.append(t0)
        for name, by_cta in d.items():
            first = np.array([min(v) for v in by_cta.values()], np.float64) - t0
            last = np.array([max(v) for v in by_cta.values()], np.float64) - t0
            ph = phases.setdefault(name, {"med": [], "med_last": [], "latest": [], "ctas": []})
            ph["med"].append(float(np.median(first)))
            ph["med_last"].append(float(np.median(last)))
            ph["latest"].append(float(last.max()))
            ph["ctas"].append(len(by_cta))
    period = np.diff(np.array(starts, np.float64))
    out = {"launches": len(starts),
           "period_us_median": round(float(np.median(period)) / 1e3, 3) if period.size else None}
    for name in [v for v in EVENTS.values() if v in phases]:
        ph = phases[name]
        out[name] = {"median_cta_us": round(statistics.median(ph["med"]) / 1e3, 3),
                     "median_cta_last_us": round(statistics.median(ph["med_last"]) / 1e3, 3),
                     "latest_cta_us": round(statistics.median(ph["latest"]) / 1e3, 3),
                     "ctas": int(statistics.median(ph["ctas"]))}
    return out


def main(argv=None):
    args = parse(argv)
    lib = load_trace_lib(args.lib)
    import torch
    from . import attention as A
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib.fr_set_launch_overlap(0 if args.no_overlap else 1)
    call = (build_cfg2 if args.workload == "cfg2" else build_cfg3)(torch, args, A, dev)
    stream = torch.cuda.Stream(dev)
    ga = gb = gc = None
    if args.gemm:
        ga = torch.randn(4096, 4096, dtype=torch.float16, device=dev)
        gb = torch.randn(4096, 4096, dtype=torch.float16, device=dev)
        gc = torch.empty_like(ga)

    def step(s):
        for l in range(args.layers):
            if args.gemm:
                torch.matmul(ga, gb, out=gc)
            call(l, s)

    with torch.cuda.stream(stream):
        step(stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
    torch.cuda.synchronize()
    buf = torch.zeros(MAX_CTAS * PER_CTA * REC.itemsize, dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    assert lib.fr_trace_attach(buf.data_ptr()) == 0
    with torch.cuda.stream(stream):
        for i in range(args.replays):
            flush.fill_(i)
            g.replay()
    torch.cuda.synchronize()
    lib.fr_trace_attach(None)
    allrec = np.frombuffer(buf.cpu().numpy().tobytes(), dtype=REC).reshape(MAX_CTAS, PER_CTA)
    per_cta = records_by_cta(allrec)
    n = int(sum(r.size for r in per_cta.values()))
    res = summarise(per_cta)
    if args.dump:
        np.savez_compressed(args.dump, **{f"cta{c}": r for c, r in per_cta.items()})
    res["workload"] = {"name": args.workload, "kv_len": args.kv if args.workload == "cfg2" else None,
                       "shard": args.shard if args.workload == "cfg3" else None,
                       "layers": args.layers, "replays": args.replays,
                       "launch_overlap": not args.no_overlap, "gemm_between_calls": args.gemm,
                       "records": int(n)}
    print(json.dumps(res))


if __name__ == "__main__":
    sys.exit(main())
