"""Multi-GPU sharding of the decode path: one process per GPU, torch.distributed
for the plumbing (NCCL between GPUs; gloo works for the host-side tests).

Every (sequence, KV head, split) unit of the decode is independent and KV
ranges combine by an associative log-sum-exp merge, so three layouts cover
the workloads:

* **DP by batch** (``plan_batch``): each rank owns whole sequences, balanced
  by total context length (greedy longest-processing-time).  No exchange on
  the hot path; ``gather_rows`` collects outputs when a caller wants them.
* **TP by KV head** (``plan_kv_heads``): each rank owns ``Hk / world`` KV
  heads and their ``G`` query heads; its cache holds only those heads, so the
  local decode is the ordinary single-GPU call on a narrower cache and the
  output stays head-sharded.
* **SP split-KV** (``plan_sequence`` / ``sp_decode``): each rank owns one
  page-aligned token range of every sequence (its own cache blocks and block
  table), runs Stage1 + Stage2 over it to one (O, LSE) per (b, h), all-gathers
  the ``[B, Hq, D+1]`` partials (NCCL over NVLink), and merges them with
  ``tqb_merge_partials``.

The reference implementation has no multi-GPU path; the exchange and merge
follow the single-GPU split merge (reference baseline/stage2.py:37-52).
"""

from __future__ import annotations

import ctypes

import heapq
import math
from typing import Optional, Sequence

import torch

from .layout import BLOCK_SIZE, HEAD_DIM


# ---------------------------------------------------------------------------
# plans (host only)
# ---------------------------------------------------------------------------


def plan_batch(seq_lens: Sequence[int], world: int) -> list[list[int]]:
    """Sequence indices of each rank, balanced by total context length
    (longest first onto the least loaded rank; ties to the lower rank).
    Every sequence lands on exactly one rank, in ascending order per rank."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(seq_lens)), key=lambda b: (-int(seq_lens[b]), b))
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for b in order:
        load, r = heapq.heappop(heap)
        out[r].append(b)
        heapq.heappush(heap, (load + int(seq_lens[b]), r))
    return [sorted(x) for x in out]


def plan_kv_heads(num_q_heads: int, num_kv_heads: int, world: int) -> list[tuple[int, int, int, int]]:
    """Per rank ``(kv0, kv1, q0, q1)``: the KV heads [kv0, kv1) and their query
    heads [q0, q1) (query head h belongs to KV head h // G)."""
    if num_kv_heads % world or num_q_heads % num_kv_heads:
        raise ValueError(f"cannot split {num_kv_heads} KV heads ({num_q_heads} query heads) over {world} ranks")
    per = num_kv_heads // world
    g = num_q_heads // num_kv_heads
    return [(r * per, (r + 1) * per, r * per * g, (r + 1) * per * g) for r in range(world)]


def plan_sequence(seq_len: int, world: int, block_size: int = BLOCK_SIZE) -> list[tuple[int, int]]:
    """Token ranges ``[t0, t1)`` of one sequence, one per rank: contiguous,
    page-aligned (so every page lives on one rank) and as even as the page
    granularity allows.  Trailing ranks may be empty."""
    pages = math.ceil(seq_len / block_size)
    per = math.ceil(pages / world) if pages else 0
    out = []
    for r in range(world):
        t0 = min(r * per * block_size, seq_len)
        t1 = min((r + 1) * per * block_size, seq_len)
        out.append((t0, t1))
    return out


def sp_shard(block_table: torch.Tensor, seq_lens: Sequence[int], world: int, rank: int,
             block_size: int = BLOCK_SIZE) -> tuple[torch.Tensor, torch.Tensor, list[tuple[int, int]]]:
    """Rank ``rank``'s share of a global paged layout under SP: its block
    table (the page columns of its token range, left-aligned), its local
    sequence lengths (int32) and its token ranges.  Block ids are left as in
    the global table; a deployment gives each rank a cache holding only its
    own pages and renumbers them."""
    ranges = [plan_sequence(int(n), world, block_size)[rank] for n in seq_lens]
    lens = [t1 - t0 for t0, t1 in ranges]
    width = max(1, max(math.ceil(n / block_size) for n in lens) if lens else 1)
    bt = torch.zeros(block_table.shape[0], width, dtype=torch.int32, device=block_table.device)
    for b, (t0, t1) in enumerate(ranges):
        p0, p1 = t0 // block_size, math.ceil(t1 / block_size)
        if p1 > p0:
            bt[b, : p1 - p0] = block_table[b, p0:p1]
    return bt, torch.tensor(lens, dtype=torch.int32, device=block_table.device), ranges


# ---------------------------------------------------------------------------
# exchange
# ---------------------------------------------------------------------------


def _world(group) -> tuple[int, int]:
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def pack_partial(out: torch.Tensor, lse: torch.Tensor) -> torch.Tensor:
    """(O [B, Hq, D], LSE [B, Hq]) -> one contiguous ``[B, Hq, D+1]`` row set."""
    return torch.cat([out, lse.unsqueeze(-1)], dim=-1).contiguous()


def gather_partials(partial: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather every rank's ``[B, Hq, D+1]`` partial into ``[G, B, Hq, D+1]``
    (rank order).  One collective; NCCL for CUDA tensors, gloo for CPU."""
    world, _ = _world(group)
    if world == 1:
        return partial.unsqueeze(0).contiguous()
    import torch.distributed as dist

    out = torch.empty((world * partial.shape[0],) + tuple(partial.shape[1:]), dtype=partial.dtype,
                      device=partial.device)
    dist.all_gather_into_tensor(out, partial.contiguous(), group=group)
    return out.view((world,) + tuple(partial.shape))


def gather_rows(local: torch.Tensor, counts: Sequence[int], group=None) -> torch.Tensor:
    """Concatenate every rank's leading-dimension rows (rank r contributes
    ``counts[r]`` rows) on every rank, for DP outputs.  Ranks pad to the
    largest count so one all-gather suffices."""
    world, _ = _world(group)
    if world == 1:
        return local
    import torch.distributed as dist

    m = max(counts)
    pad = torch.zeros((m,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    buf = torch.empty((world * m,) + tuple(pad.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, pad, group=group)
    buf = buf.view((world,) + tuple(pad.shape))
    return torch.cat([buf[r, : counts[r]] for r in range(world)], dim=0)


# ---------------------------------------------------------------------------
# decode drivers (GPU)
# ---------------------------------------------------------------------------


def local_partial(q_rot: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                  seq_lens: torch.Tensor, centroids: torch.Tensor, num_splits: int, *,
                  layout: str = "soa", mid_o: Optional[torch.Tensor] = None,
                  attn_scale: Optional[float] = None) -> torch.Tensor:
    """Stage1 + Stage2 over this rank's KV range: ``[B, Hq, D+1]`` (O, LSE).
    A sequence with no local token gets LSE = -inf, which the merge skips."""
    from . import ops

    B, Hq, D = q_rot.shape
    if mid_o is None:
        mid_o = torch.empty(B, Hq, num_splits, D + 1, device=q_rot.device)
    out = torch.empty(B, Hq, D, device=q_rot.device)
    lse = torch.empty(B, Hq, device=q_rot.device)
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout=layout, attn_scale=attn_scale)
    ops.stage2(mid_o, seq_lens, out, lse)
    return pack_partial(out, lse)


def sp_decode(q_rot: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
              seq_lens: torch.Tensor, centroids: torch.Tensor, *, local_splits: int = 16,
              layout: str = "soa", group=None, attn_scale: Optional[float] = None,
              output: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None):
    """Sequence-parallel decode step on this rank: local Stage1 (``local_splits``
    splits) + Stage2 over the rank's own pages (``kv_cache``, ``block_table``,
    ``seq_lens`` are the local shard), all-gather of the partials, and the
    cross-range merge.  Every rank returns the full (O [B, Hq, D], LSE [B, Hq])."""
    from . import ops

    part = local_partial(q_rot, kv_cache, block_table, seq_lens, centroids, local_splits, layout=layout,
                         attn_scale=attn_scale)
    parts = gather_partials(part, group)
    B, Hq, D = q_rot.shape
    if output is None:
        output = torch.empty(B, Hq, D, device=q_rot.device)
    if lse is None:
        lse = torch.empty(B, Hq, device=q_rot.device)
    ops.merge_partials(parts, output, lse)
    return output, lse


def sp_decode_p2p(exchange: "P2PExchange", q_rot: torch.Tensor, kv_cache: torch.Tensor,
                  block_table: torch.Tensor, seq_lens: torch.Tensor, centroids: torch.Tensor, *,
                  local_splits: int = 16, layout: str = "soa", attn_scale: Optional[float] = None,
                  mid_o: Optional[torch.Tensor] = None, output: Optional[torch.Tensor] = None,
                  lse: Optional[torch.Tensor] = None):
    """``sp_decode`` with the exchange over peer memory: local Stage1, then
    ``exchange.step`` (Stage2 rows straight into every rank's buffer, merge of
    all ranks' rows).  Every rank returns the full (O [B, Hq, D], LSE [B, Hq])."""
    from . import ops

    B, Hq, D = q_rot.shape
    if mid_o is None:
        mid_o = torch.empty(B, Hq, local_splits, D + 1, device=q_rot.device)
    if output is None:
        output = torch.empty(B, Hq, D, device=q_rot.device)
    if lse is None:
        lse = torch.empty(B, Hq, device=q_rot.device)
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout=layout, attn_scale=attn_scale)
    return exchange.step(mid_o, seq_lens, output, lse)


class P2PExchange:
    """Per-rank state of the sequence-parallel exchange over peer memory
    (``tqb_sp_exchange`` / ``tqb_sp_merge``): this rank's exchange buffer,
    every rank's buffer mapped into this process (CUDA IPC handles swapped
    over the process group once), and the step epoch.  ``step`` replaces
    Stage2 + all-gather + merge: each rank's merged rows go straight into
    every rank's buffer over NVLink and every rank merges the G rows.

    ``emulated(world, ...)`` builds the ``world`` ranks of one process on one
    GPU (the buffers are local; ranks are stepped one after another), for
    testing the data path without IPC.

    ``device_epochs=True`` keeps the step epoch in the exchange buffer on the
    device (epoch 0 in the C calls): ``step`` then passes no per-step value,
    so it can be recorded into a CUDA graph with Stage1 and replayed."""

    def __init__(self, batch: int, num_q_heads: int, device: torch.device, group=None, *,
                 device_epochs: bool = False, _local: Optional[dict] = None):
        from . import _lib

        self._lib = _lib.load()
        self.device = torch.device(device)
        self.cap_rows = batch * num_q_heads
        self.device_epochs = device_epochs
        self.epoch = 0
        self._imported = []
        self._owned = None
        if _local is not None:  # emulated rank: buffers shared inside one process
            self.world, self.rank, self.buffers = _local["world"], _local["rank"], _local["buffers"]
            return
        self.world, self.rank = _world(group)
        self.group = group
        nbytes = self._lib.tqb_p2p_buffer_bytes(self.world, self.cap_rows)
        _lib.check(_lib.TQB_OK if nbytes > 0 else _lib.TQB_ERR_INVALID_ARG)
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self._lib.tqb_p2p_alloc(nbytes, ctypes.byref(own)))
        self._owned = own.value
        buffers = [None] * self.world
        buffers[self.rank] = own.value
        if self.world > 1:
            import torch.distributed as dist

            h = (ctypes.c_char * _lib.TQB_IPC_HANDLE_BYTES)()
            _lib.check(self._lib.tqb_ipc_export(ctypes.c_void_p(own.value), h))
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h), group=group)
            with torch.cuda.device(self.device):
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    ptr = ctypes.c_void_p()
                    hr = (ctypes.c_char * _lib.TQB_IPC_HANDLE_BYTES).from_buffer_copy(handles[r])
                    _lib.check(self._lib.tqb_ipc_import(hr, ctypes.byref(ptr)))
                    self._imported.append(ptr.value)
                    buffers[r] = ptr.value
        self.buffers = buffers

    @classmethod
    def emulated(cls, world: int, batch: int, num_q_heads: int, device: torch.device, *,
                 device_epochs: bool = False) -> list["P2PExchange"]:
        from . import _lib

        lib = _lib.load()
        nbytes = lib.tqb_p2p_buffer_bytes(world, batch * num_q_heads)
        bufs = []
        with torch.cuda.device(device):
            for _ in range(world):
                p = ctypes.c_void_p()
                _lib.check(lib.tqb_p2p_alloc(nbytes, ctypes.byref(p)))
                bufs.append(p.value)
        ranks = [cls(batch, num_q_heads, device, device_epochs=device_epochs,
                     _local={"world": world, "rank": r, "buffers": bufs}) for r in range(world)]
        ranks[0]._owned_list = bufs  # freed by ranks[0].close()
        return ranks

    def step(self, mid_o: torch.Tensor, seq_lens: torch.Tensor, output: torch.Tensor,
             lse: Optional[torch.Tensor] = None, *, num_splits_per_seq: Optional[torch.Tensor] = None,
             stream: Optional[int] = None):
        """This rank's Stage2 rows to every rank (``send``), then the merge of
        all ranks' rows into ``output [B, Hq, D]`` and ``lse [B, Hq]`` (``recv``)."""
        self.send(mid_o, seq_lens, num_splits_per_seq=num_splits_per_seq, stream=stream)
        return self.recv(output, lse, stream=stream)

    def _stream(self, stream):
        return stream if stream is not None else torch.cuda.current_stream(self.device).cuda_stream

    def send(self, mid_o: torch.Tensor, seq_lens: torch.Tensor, *,
             num_splits_per_seq: Optional[torch.Tensor] = None, stream: Optional[int] = None) -> None:
        """Stage2 of this rank's splits, each row stored into every rank's
        buffer, and the new epoch published (``tqb_sp_exchange``)."""
        from . import _lib

        B, Hq, S, D1 = mid_o.shape
        if B * Hq > self.cap_rows:
            raise _lib.TqbError(_lib.TQB_ERR_INVALID_ARG, "batch * num_q_heads exceeds the exchange capacity")
        self.epoch += 1
        self._shape = (B, Hq, D1 - 1)
        a = _lib.SpExchangeArgs()
        s2 = a.stage2
        s2.mid_o = mid_o.data_ptr()
        s2.mid_stride_b, s2.mid_stride_h, s2.mid_stride_s = mid_o.stride(0), mid_o.stride(1), mid_o.stride(2)
        s2.seq_lens = seq_lens.data_ptr()
        if num_splits_per_seq is not None:
            s2.num_splits_per_seq = num_splits_per_seq.data_ptr()
        s2.batch, s2.num_q_heads, s2.head_dim, s2.num_splits = B, Hq, D1 - 1, S
        a.rank, a.world, a.cap_rows = self.rank, self.world, self.cap_rows
        a.epoch = 0 if self.device_epochs else self.epoch
        for r, p in enumerate(self.buffers):
            a.buffers[r] = p
        with torch.cuda.device(self.device):
            _lib.check(self._lib.tqb_sp_exchange(ctypes.byref(a), ctypes.c_void_p(self._stream(stream))))

    def recv(self, output: torch.Tensor, lse: Optional[torch.Tensor] = None, *, stream: Optional[int] = None):
        """Wait for every rank's rows of the current epoch and merge them
        (``tqb_sp_merge``)."""
        from . import _lib

        B, Hq, D = self._shape
        m = _lib.SpMergeArgs()
        m.buffer, m.world, m.batch, m.num_q_heads, m.head_dim = self.buffers[self.rank], self.world, B, Hq, D
        m.cap_rows = self.cap_rows
        m.epoch = 0 if self.device_epochs else self.epoch
        m.output, m.out_stride_b, m.out_stride_h = output.data_ptr(), output.stride(0), output.stride(1)
        if lse is not None:
            m.lse, m.lse_stride_b = lse.data_ptr(), lse.stride(0)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.tqb_sp_merge(ctypes.byref(m), ctypes.c_void_p(self._stream(stream))))
        return output, lse

    def close(self) -> None:
        """Unmap the other ranks' buffers and free this rank's (collective:
        every rank calls it)."""
        from . import _lib

        torch.cuda.synchronize(self.device)
        if self._owned is not None and self.world > 1:
            import torch.distributed as dist

            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._imported:
                self._lib.tqb_ipc_close(ctypes.c_void_p(p))
            self._imported = []
            if self._owned is not None and self.world > 1:
                import torch.distributed as dist

                dist.barrier(group=self.group)
            if self._owned is not None:
                self._lib.tqb_p2p_free(ctypes.c_void_p(self._owned))
                self._owned = None
            for p in getattr(self, "_owned_list", []):
                self._lib.tqb_p2p_free(ctypes.c_void_p(p))
            self._owned_list = []


def tp_shard_cache(kv_cache: torch.Tensor, world: int, rank: int, layout: str = "soa") -> torch.Tensor:
    """Rank ``rank``'s cache under TP by KV head: the same blocks holding only
    its ``Hk / world`` heads, as a new ``[num_blocks, 16, Hk_local, 134]``
    uint8 tensor.  SoA blocks are rebuilt (data rows ``[16][Hk][128]`` and the
    metadata ``[Hk][3][16]`` fp16 both narrowed to the rank's heads); an AoS
    cache is a plain slice of its head dimension."""
    nb, bs, hk, slot = kv_cache.shape
    kv0, kv1, _, _ = plan_kv_heads(hk, hk, world)[rank]
    if layout == "aos":
        return kv_cache[:, :, kv0:kv1].contiguous()
    raw = kv_cache.reshape(nb, -1)
    data = raw[:, : bs * hk * HEAD_DIM].reshape(nb, bs, hk, HEAD_DIM)[:, :, kv0:kv1]
    meta = raw[:, bs * hk * HEAD_DIM : bs * hk * slot].reshape(nb, hk, 3 * bs * 2)[:, kv0:kv1]
    out = torch.cat([data.reshape(nb, -1), meta.reshape(nb, -1)], dim=1)
    return out.reshape(nb, bs, kv1 - kv0, slot).contiguous()


def tp_shard_query(q_rot: torch.Tensor, num_kv_heads: int, world: int, rank: int) -> torch.Tensor:
    """Rank ``rank``'s query heads under TP by KV head (a view)."""
    kv0, kv1, q0, q1 = plan_kv_heads(q_rot.shape[1], num_kv_heads, world)[rank]
    return q_rot[:, q0:q1]


__all__ = ["plan_batch", "plan_kv_heads", "plan_sequence", "sp_shard", "pack_partial", "gather_partials",
           "gather_rows", "local_partial", "sp_decode", "tp_shard_cache", "tp_shard_query"]
