"""Multi-GPU execution of the attention path (one process per GPU).

Two schemes, both new relative to the reference (which is single-GPU,
`docs/flux_server.md:84-88`):

* (batch x head) partition, no collective. The B*H (b, h) units are
  independent, so rank r of N computes the contiguous unit range
  [r*U/N, (r+1)*U/N) straight from strided views of the full tensors and
  writes its slice of O. `partition_units` / `head_split_attention`.

* Sequence-sharded attention for long sequences. Rank r holds tokens
  [r*S/P, (r+1)*S/P). It normalises and rotates its own Q/K once (global
  RoPE rows and global txt/img gain split), then runs P steps; in step t it
  attends with its Q to the K/V block of rank (r - t) mod P (fp32 partial O
  + LSE), merged into the running result by log-sum-exp in the attention
  kernel's epilogue (LLMR_MERGE). `RingAttention`, with two transports for
  the K/V blocks:
  - "copy": every rank exports its fp16 Q/K/V block (CUDA IPC) once; after
    a barrier that follows all prologues, each rank pulls the P-1 other
    blocks straight from their owners on the copy engines, in step order,
    on a side stream, while the attention kernel runs on all SMs. NVSwitch
    gives every pair full bandwidth, so no block is passed on hop by hop.
    Received blocks are stored so that each head's keys of all blocks are
    contiguous, and the kernel covers groups of arrived blocks in one launch
    (`ring_groups`: own block, then 1, 1, 2, 3, ... blocks). A second barrier
    after the pulls lets owners overwrite their block in the next call.
  - "nccl": the classic ring: the current block goes to rank r+1 and the
    next one comes from rank r-1 by NCCL P2P (batch_isend_irecv) each step.

The ring's schedule and merge are plain host logic over pluggable ops, so
they are exercised on CPU with gloo ranks as well as on GPUs with NCCL.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import llmr_attn as L


# ---------------------------------------------------------------- head split

def partition_units(batch: int, n_heads: int, world: int, rank: int) -> List[Tuple[int, int, int]]:
    """Rank `rank`'s share of the batch*n_heads (b, h) units as runs
    (b, h0, h1) inside single batch elements. Shares differ by at most one
    unit (Z-Image's 60 units on 8 GPUs: four ranks get 8, four get 7)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    units = batch * n_heads
    lo = rank * units // world
    hi = (rank + 1) * units // world
    runs = []
    u = lo
    while u < hi:
        b, h0 = divmod(u, n_heads)
        h1 = min(n_heads, h0 + (hi - u))
        runs.append((b, h0, h1))
        u += h1 - h0
    return runs


def head_split_attention(ctx: "L.Context", q, k, v, o, cfg: "L.AttnConfig", *, batch: int,
                         seq_len: int, rank: int, world: int, q_gain=None, k_gain=None,
                         cos=None, sin=None) -> List[Tuple[int, int, int]]:
    """This rank's (b, h) units of the fused op. q/k/v are the full BSHD
    [B,S,H,D] tensors (or views of them), o the full [B,S,H*D] output; only
    this rank's head slices of o are written. No communication."""
    H, D = cfg.n_heads, cfg.head_dim
    if cfg.layout != L.BSHD:
        raise ValueError("head_split_attention expects BSHD inputs")
    runs = partition_units(batch, H, world, rank)
    for b, h0, h1 in runs:
        sub = L.AttnConfig(**{**cfg.__dict__, "n_heads": h1 - h0})
        st = {"q_row_stride": q.stride(1), "k_row_stride": k.stride(1),
              "v_row_stride": v.stride(1), "q_head_stride": q.stride(2),
              "k_head_stride": k.stride(2), "v_head_stride": v.stride(2),
              "o_row_stride": o.stride(1)}
        L.attention_fused(ctx, q[b, :, h0:h1], k[b, :, h0:h1], v[b, :, h0:h1],
                          o[b, :, h0 * D:h1 * D], sub, batch=1, seq_len=seq_len,
                          q_gain=q_gain, k_gain=k_gain, cos=cos, sin=sin, strides=st)
    return runs


# ---------------------------------------------------------------------- ring

class RingOps:
    """The device steps of the ring, on the library's CUDA kernels."""

    def __init__(self, ctx: "L.Context", cfg: "L.AttnConfig", seq_local: int,
                 row_offset: int, copy_streams: int = 1):
        self.ctx, self.cfg, self.S, self.off = ctx, cfg, seq_local, row_offset
        self.n_copy = max(1, copy_streams)
        self.part_cfg = L.AttnConfig(n_heads=cfg.n_heads, head_dim=cfg.head_dim,
                                     scale=cfg.scale, layout=L.BHSD)

    def empty(self, shape, dtype, device):
        import torch
        return torch.empty(shape, dtype=dtype, device=device)

    def prologue(self, q, k, v, qkv_out, q_gain, k_gain, cos, sin):
        pc = L.AttnConfig(**{**self.cfg.__dict__, "rope_row_offset": self.off})
        L.attention_prologue(self.ctx, q, k, v, qkv_out, pc, batch=1, seq_len=self.S,
                             q_gain=q_gain, k_gain=k_gain, cos=cos, sin=sin)

    def partial(self, qh, kh, vh, o, lse, merge):
        """Attention of this rank's Q [H, S, D] against the keys of kh / vh
        ([H, T, D] views, T a multiple of the shard length, any head stride)
        into (o, lse); with merge, folded into the result already there
        (log-sum-exp merge in the kernel's epilogue)."""
        st = {"k_row_stride": kh.stride(1), "k_head_stride": kh.stride(0),
              "v_row_stride": vh.stride(1), "v_head_stride": vh.stride(0)}
        L.attention_fused(self.ctx, qh, kh, vh, o, self.part_cfg, batch=1, seq_len=self.S,
                          lse=lse, merge=merge, kv_len=kh.shape[1], strides=st)

    def finalize(self, o_acc, out):
        L.convert_f32(self.ctx, o_acc, out)

    # -- "copy" transport: peer blocks on the copy engines ----------------------

    def share(self, shape, dtype, device, rank, world, group):
        """Allocates this rank's Q/K/V block as an exportable buffer and maps
        every other rank's (collective over `group`)."""
        import torch
        import torch.distributed as dist
        n = 1
        for x in shape:
            n *= int(x)
        esize = torch.empty((), dtype=dtype).element_size()
        self.own = L.DeviceBuffer(self.ctx, n * esize)
        handles = [None] * world
        dist.all_gather_object(handles, self.own.export(), group=group)
        self.peers = [None if r == rank else L.PeerMapping(self.ctx, handles[r])
                      for r in range(world)]
        self.kv_offset = (n // shape[0]) * esize          # bytes of the Q part
        self.kv_bytes = 2 * self.kv_offset
        self.group = group
        self.compute = torch.cuda.current_stream()
        # Side streams for the pulls: copies on different streams run on
        # different copy engines at once. comm[0] also carries the barriers.
        self.comm_streams = [torch.cuda.Stream() for _ in range(self.n_copy)]
        self.comm = self.comm_streams[0]
        self.tok = torch.zeros(1, device=device)
        self.released = None
        return self.own.tensor(shape, dtype)

    def _barrier_on_comm(self):
        import torch
        import torch.distributed as dist
        with torch.cuda.stream(self.comm):
            dist.all_reduce(self.tok, group=self.group)

    def wait_released(self):
        """The compute stream waits until every rank has finished reading this
        rank's block of the previous call."""
        if self.released is not None:
            self.compute.wait_event(self.released)

    def sync_peers(self):
        """Barrier (on the side stream) after this rank's compute so far, i.e.
        after every rank's prologue: peers' blocks are complete after it."""
        self.comm.wait_stream(self.compute)
        self._barrier_on_comm()
        for st in self.comm_streams[1:]:
            st.wait_stream(self.comm)

    def fetch(self, src_rank, slot, kv_recv):
        """Copies rank src_rank's K/V block ([2][H][S][D]) into slot `slot` of
        kv_recv ([2][H][n_slots*S][D], each head's keys of all slots
        contiguous) on the side stream, one 2-D copy per K and V; returns the
        event the compute stream waits for before using it."""
        import torch
        _, H, T, D = kv_recv.shape
        S = self.S
        esize = kv_recv.element_size()
        row = S * D * esize                       # one head of one block
        # K and V, each cut into head ranges, spread over the side streams
        parts = []
        per = max(1, (2 * len(self.comm_streams)) // 2)
        for i in range(2):
            for c in range(per):
                h0, h1 = c * H // per, (c + 1) * H // per
                if h1 > h0:
                    parts.append((i, h0, h1))
        events = []
        for n, (i, h0, h1) in enumerate(parts):
            st = self.comm_streams[n % len(self.comm_streams)]
            dst = kv_recv[i].data_ptr() + h0 * T * D * esize + slot * row
            src = self.peers[src_rank].ptr + self.kv_offset + (i * H + h0) * row
            L.copy2d_async(self.ctx, dst, T * D * esize, src, row, row, h1 - h0, st)
        for st in self.comm_streams:
            ev = torch.cuda.Event()
            ev.record(st)
            events.append(ev)
        return events

    def wait(self, events):
        for ev in events:
            self.compute.wait_event(ev)

    def release(self):
        """Barrier after this rank's pulls: when every rank has passed it, no
        rank reads this rank's block any more."""
        import torch
        for st in self.comm_streams[1:]:
            self.comm.wait_stream(st)
        self._barrier_on_comm()
        self.released = torch.cuda.Event()
        self.released.record(self.comm)

    def close(self):
        for m in getattr(self, "peers", []):
            if m is not None:
                m.close()
        if getattr(self, "own", None) is not None:
            self.own.close()
            self.own = None


@dataclass
class RingBuffers:
    qkv: object      # fp16 [3, H, S_loc, D] (Q', K', V' of this rank)
    kv_nxt: object   # fp16 [2, H, S_loc, D] (receive buffer)
    o_acc: object    # fp32 [S_loc, H*D]
    lse_acc: object  # fp32 [H, S_loc]


class RingAttention:
    """Sequence-sharded attention over a torch.distributed group; the K/V
    blocks move by `transport` ("copy" or "nccl", see the module notes)."""

    def __init__(self, ops, n_heads: int, head_dim: int, seq_total: int, rank: int,
                 world: int, device, group=None, qkv_dtype=None, transport: str = "nccl"):
        import torch
        if seq_total % world:
            raise ValueError("seq_total must divide evenly over the ring")
        if transport not in ("nccl", "copy"):
            raise ValueError(f"unknown transport {transport!r}")
        self.ops, self.rank, self.world, self.group = ops, rank, world, group
        self.transport = transport
        self.S = seq_total // world
        H, D, S = n_heads, head_dim, self.S
        dt = qkv_dtype or torch.float16
        if transport == "copy":
            qkv = ops.share((3, H, S, D), dt, device, rank, world, group)
            nxt = ops.empty((2, H, max(world - 1, 1) * S, D), dt, device)
        else:
            qkv = ops.empty((3, H, S, D), dt, device)
            nxt = ops.empty((2, H, S, D), dt, device)
        self.buf = RingBuffers(
            qkv=qkv, kv_nxt=nxt,
            o_acc=ops.empty((S, H * D), torch.float32, device),
            lse_acc=ops.empty((H, S), torch.float32, device))

    def close(self) -> None:
        if hasattr(self.ops, "close"):
            self.ops.close()

    def forward(self, q, k, v, out, q_gain=None, k_gain=None, cos=None, sin=None) -> None:
        """q/k/v: this rank's token shard [1, S_loc, H, D]; out: [1, S_loc, H*D]."""
        if self.transport == "copy":
            return self._forward_copy(q, k, v, out, q_gain, k_gain, cos, sin)
        import torch.distributed as dist
        b = self.buf
        self.ops.prologue(q, k, v, b.qkv, q_gain, k_gain, cos, sin)
        qh = b.qkv[0]
        kv_cur, kv_nxt = b.qkv[1:3], b.kv_nxt
        nxt_rank = (self.rank + 1) % self.world
        prv_rank = (self.rank - 1) % self.world
        for t in range(self.world):
            reqs = None
            if t < self.world - 1:
                reqs = dist.batch_isend_irecv([
                    dist.P2POp(dist.isend, kv_cur, nxt_rank, self.group),
                    dist.P2POp(dist.irecv, kv_nxt, prv_rank, self.group)])
            self.ops.partial(qh, kv_cur[0], kv_cur[1], b.o_acc, b.lse_acc, merge=t > 0)
            if reqs is not None:
                for w in reqs:
                    w.wait()
            kv_cur, kv_nxt = kv_nxt, kv_cur
        self.ops.finalize(b.o_acc, out)

    def _forward_copy(self, q, k, v, out, q_gain, k_gain, cos, sin) -> None:
        ops, b, P, r, S = self.ops, self.buf, self.world, self.rank, self.S
        ops.wait_released()
        ops.prologue(q, k, v, b.qkv, q_gain, k_gain, cos, sin)
        events = []
        if P > 1:
            ops.sync_peers()
            # slot t-1 receives the block of rank (r - t) mod P, in step order
            events = [ops.fetch((r - t) % P, t - 1, b.kv_nxt) for t in range(1, P)]
        qh = b.qkv[0]
        ops.partial(qh, b.qkv[1], b.qkv[2], b.o_acc, b.lse_acc, merge=False)
        for a, n in ring_groups(P - 1):
            ops.wait(events[a + n - 1])   # copies run in order on one stream
            ops.partial(qh, b.kv_nxt[0][:, a * S:(a + n) * S], b.kv_nxt[1][:, a * S:(a + n) * S],
                        b.o_acc, b.lse_acc, merge=True)
        if P > 1:
            ops.release()
        ops.finalize(b.o_acc, out)


def ring_groups(n: int) -> List[Tuple[int, int]]:
    """Received blocks 0..n-1 as consecutive (first, count) groups of
    Fibonacci sizes (1, 1, 2, 3, 5, ...; the last group takes what is left):
    one attention launch per group. A group only needs blocks that arrived
    while the previous groups were computed, as long as computing one block
    takes about as long as pulling one, so the kernel never waits for the
    copy engines; the growing sizes keep the number of launches small.
    n=7 -> [(0, 1), (1, 1), (2, 2), (4, 3)]."""
    groups, i, a, b = [], 0, 1, 1
    while i < n:
        take = min(a, n - i)
        groups.append((i, take))
        i += take
        a, b = b, a + b
    return groups
