"""Multi-GPU partitioning of decode attention, one process per GPU.

The reference is single-GPU (its decode loop is one sequence on device 0,
runtime/main.cpp:173-228); these are the two partitionings the engine adds:

* Batched decode (no collective).  The unit of work is a (sequence, kv head)
  pair: its K/V rows and its G query heads live on one GPU, which writes the
  matching disjoint slice of the output.  Units are assigned
  longest-processing-time first by token count, so ranks get equal KV bytes.

* One long sequence (one exchange).  The KV range [0, kv_len) is cut into P
  contiguous ranges; each rank holds only its range and computes one
  log-sum-exp state (m, l, acc[D]) per query head over it
  (fr_decode_attn_partial).  One all-gather of H*(2+D) fp32 per rank
  (14,560 B for the Qwen2-7B shape) brings every rank's state to every rank,
  and the LSE merge (fr_lse_merge_strided, reading the gathered buffer in
  place) produces the fp16 output.  Merging is associative, so every rank
  ends with the same output regardless of the order states arrive.

The compute callables are injectable so the partition/exchange logic runs
under the gloo backend on CPU with the numpy oracle in tests.
"""
from __future__ import annotations

import heapq
from typing import Callable, Sequence


def lpt_assign(weights: Sequence[int], world: int) -> list[list[int]]:
    """Greedy longest-processing-time assignment of units to `world` ranks.

    Units are taken by decreasing weight (ties by index) and each goes to the
    currently lightest rank (ties by rank id).  Returns, per rank, the sorted
    unit indices.  Deterministic, so every rank computes the same plan.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(weights)), key=lambda i: (-int(weights[i]), i))
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(weights[i]), r))
    return [sorted(u) for u in out]


def batched_units(kv_lens: Sequence[int], num_kv_heads: int) -> list[tuple[int, int, int]]:
    """(sequence, kv_head, tokens) for every unit of a batch."""
    return [(b, h, int(n)) for b, n in enumerate(kv_lens) for h in range(num_kv_heads)]


def shard_batched(kv_lens: Sequence[int], num_kv_heads: int, world: int):
    """Per rank, the list of (sequence, kv_head, tokens) units it owns."""
    units = batched_units(kv_lens, num_kv_heads)
    plan = lpt_assign([u[2] for u in units], world)
    return [[units[i] for i in idx] for idx in plan]


def kv_ranges(kv_len: int, world: int, align: int = 64) -> list[tuple[int, int]]:
    """Contiguous [begin, end) ranges covering [0, kv_len), one per rank.

    Boundaries are multiples of `align` positions (one pipeline tile), sizes
    differ by at most one tile; trailing ranks may be empty when kv_len is
    short.
    """
    if world <= 0 or kv_len < 0:
        raise ValueError("bad kv_len / world")
    tiles = -(-kv_len // align)
    base, extra = divmod(tiles, world)
    out = []
    t = 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        b = min(t * align, kv_len)
        e = min((t + n) * align, kv_len)
        out.append((b, e))
        t += n
    return out


class LongContextDecoder:
    """KV-range-sharded decode of one sequence across the ranks of `group`.

    partial_fn(q, k_local, v_local, local_len, state_ml, state_acc)
        writes this rank's state: state_ml [H, 2], state_acc [H, D] fp32
        (views into one contiguous [H*(2+D)] buffer).
    merge_fn(gathered, world, out)
        merges the gathered [world, H*(2+D)] buffer into out [H, D].
    The defaults are the CUDA entry points; tests pass numpy versions.
    """

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, device, group=None,
                 partial_fn: Callable | None = None, merge_fn: Callable | None = None):
        import torch
        import torch.distributed as dist

        self.torch = torch
        self.dist = dist
        self.group = group
        self.H, self.Hkv, self.D = num_heads, num_kv_heads, head_dim
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.state_elems = num_heads * (2 + head_dim)
        self.local = torch.empty(self.state_elems, dtype=torch.float32, device=device)
        self.gathered = torch.empty((self.world, self.state_elems), dtype=torch.float32,
                                    device=device)
        self.partial_fn = partial_fn or self._cuda_partial
        self.merge_fn = merge_fn or self._cuda_merge
        backend = dist.get_backend(group) if dist.is_initialized() else "none"
        self.use_into_tensor = backend == "nccl"

    # state_ml / state_acc as views of the packed buffer
    def views(self, buf):
        return buf[:2 * self.H].view(self.H, 2), buf[2 * self.H:].view(self.H, self.D)

    def _cuda_partial(self, q, k_local, v_local, local_len, state_ml, state_acc, stream=None):
        from . import attention as A
        A.decode_attn_partial(q, k_local if local_len else 0, v_local if local_len else 0,
                              local_len, state_ml, state_acc, self.H, self.Hkv, self.D, stream)

    def _cuda_merge(self, gathered, world, out, stream=None):
        from ._lib import check, load
        from .attention import _stream
        lib = load()
        base = gathered.data_ptr()
        check("fr_lse_merge_strided", lib.fr_lse_merge_strided(
            base, base + 2 * self.H * 4, world, out.data_ptr(), self.H, self.D,
            self.state_elems, self.state_elems, _stream(stream)))

    def exchange(self) -> None:
        if self.world == 1:
            self.gathered[0].copy_(self.local)
        elif self.use_into_tensor:
            self.dist.all_gather_into_tensor(self.gathered, self.local, group=self.group)
        else:
            self.dist.all_gather(list(self.gathered.unbind(0)), self.local, group=self.group)

    def __call__(self, q, k_local, v_local, local_len: int, out, stream=None) -> None:
        """One decode step.  `stream` (CUDA path) must be the current torch
        stream, on which the all-gather is issued."""
        ml, acc = self.views(self.local)
        if stream is None:
            self.partial_fn(q, k_local, v_local, local_len, ml, acc)
            self.exchange()
            self.merge_fn(self.gathered, self.world, out)
        else:
            self.partial_fn(q, k_local, v_local, local_len, ml, acc, stream)
            self.exchange()
            self.merge_fn(self.gathered, self.world, out, stream)


class PeerExchangeDecoder:
    """KV-range-sharded decode of one sequence with the exchange inside the
    kernel (fr_decode_attn_exchange): each rank's split kernel stores its
    (m, l, acc) states into every rank's exchange buffer over NVLink and
    merges the states it receives - no collective call on the data path.

    Set-up (collective, once): each rank allocates its buffer, the 64-byte
    CUDA IPC handles are all-gathered through `group` (any backend), and each
    rank opens the others'.  close() is collective too: it waits at a barrier
    so that no rank frees a buffer another may still write.
    """

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, device, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from ._lib import check, load

        self.lib = load()
        self.dist, self.group = dist, group
        self.H, self.Hkv, self.D = num_heads, num_kv_heads, head_dim
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.nbytes = self.lib.fr_exchange_bytes(num_heads, head_dim, self.world)
        if not self.nbytes:
            raise ValueError("unsupported exchange shape")
        with torch.cuda.device(device):
            buf = ctypes.c_void_p()
            handle = (ctypes.c_char * 64)()
            check("fr_exchange_alloc", self.lib.fr_exchange_alloc(self.nbytes, ctypes.byref(buf),
                                                                  handle))
            self.local = buf.value
            handles = [None] * self.world
            if self.world > 1:
                dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs, self.opened = [], []
            for j in range(self.world):
                if j == self.rank:
                    ptrs.append(self.local)
                    continue
                peer = ctypes.c_void_p()
                h = (ctypes.c_char * 64).from_buffer_copy(handles[j])
                check("fr_exchange_open", self.lib.fr_exchange_open(h, ctypes.byref(peer)))
                ptrs.append(peer.value)
                self.opened.append(peer.value)
        self.bufs = (ctypes.c_void_p * self.world)(*ptrs)
        self.closed = False

    def __call__(self, q, k_local, v_local, local_len: int, out, stream=None) -> None:
        from ._lib import check
        from .attention import _ptr, _stream
        check("fr_decode_attn_exchange", self.lib.fr_decode_attn_exchange(
            _ptr(q), _ptr(k_local) if local_len else None, _ptr(v_local) if local_len else None,
            local_len, _ptr(out), self.H, self.Hkv, self.D, self.bufs, self.rank, self.world,
            _stream(stream)))

    def reset(self, stream=None) -> None:
        """After a timed-out exchange: zero this rank's counters and epoch
        (every rank must do it before the next call)."""
        from ._lib import check
        from .attention import _stream
        check("fr_exchange_reset", self.lib.fr_exchange_reset(self.local, self.nbytes,
                                                              _stream(stream)))

    def close(self) -> None:
        if self.closed:
            return
        import torch
        torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier(group=self.group)
        for p in self.opened:
            self.lib.fr_exchange_close(p)
        self.lib.fr_exchange_free(self.local)
        self.closed = True
