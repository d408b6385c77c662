"""CPU: host logic of the multi-GPU schemes.

The (batch x head) partition is checked exhaustively; the sequence-sharded
ring's schedule (who sends which K/V block to whom, in which step) and its
log-sum-exp merge run as gloo ranks on CPU with exact float64 ops standing in
for the CUDA kernels, and must reproduce unsharded attention."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llmr_attn.dist import RingAttention, partition_units, ring_groups


@pytest.mark.parametrize("B,H,world", [(1, 24, 1), (1, 24, 8), (2, 30, 8), (1, 24, 7),
                                       (3, 5, 4), (1, 3, 8)])
def test_partition_units_cover_and_balance(B, H, world):
    seen = []
    sizes = []
    for r in range(world):
        runs = partition_units(B, H, world, r)
        n = 0
        for b, h0, h1 in runs:
            assert 0 <= b < B and 0 <= h0 < h1 <= H
            seen += [b * H + h for h in range(h0, h1)]
            n += h1 - h0
        sizes.append(n)
    assert sorted(seen) == list(range(B * H))
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("n", range(0, 20))
def test_ring_groups_cover_in_order(n):
    groups = ring_groups(n)
    covered = [i for a, c in groups for i in range(a, a + c)]
    assert covered == list(range(n))
    assert all(c >= 1 for _, c in groups)
    sizes = [c for _, c in groups]
    assert all(sizes[j] <= sizes[j - 1] + (sizes[j - 2] if j >= 2 else 0) for j in range(1, len(sizes)))


def test_ring_groups_eight_gpus():
    assert ring_groups(7) == [(0, 1), (1, 1), (2, 2), (4, 3)]
    assert ring_groups(1) == [(0, 1)]
    assert ring_groups(3) == [(0, 1), (1, 1), (2, 1)]


def test_partition_zimage_8_gpus():
    sizes = [sum(h1 - h0 for _, h0, h1 in partition_units(2, 30, 8, r)) for r in range(8)]
    assert sorted(sizes) == [7, 7, 7, 7, 8, 8, 8, 8]


class CpuRingOps:
    """float64 stand-ins for the CUDA steps (the kernels themselves are
    checked on the GPU); layouts match RingOps exactly."""

    def __init__(self, n_heads, head_dim, scale):
        self.H, self.D, self.scale = n_heads, head_dim, scale

    def empty(self, shape, dtype, device):
        return torch.empty(shape, dtype=torch.float64)

    def prologue(self, q, k, v, qkv_out, *unused):
        for i, t in enumerate((q, k, v)):
            qkv_out[i] = t[0].permute(1, 0, 2).to(torch.float64)

    def partial(self, qh, kh, vh, o, lse, merge):
        assert kh.shape[1] % qh.shape[1] == 0   # whole blocks of keys
        s = torch.einsum("hsd,htd->hst", qh, kh) * self.scale
        m = s.amax(-1, keepdim=True)
        p = torch.exp(s - m)
        l = p.sum(-1, keepdim=True)
        lse_t = (m + torch.log(l))[..., 0]
        o_t = torch.einsum("hst,htd->hsd", p / l, vh).permute(1, 0, 2).reshape(o.shape)
        if not merge:
            o.copy_(o_t)
            lse.copy_(lse_t)
            return
        H, D, S = self.H, self.D, o.shape[0]
        mx = torch.maximum(lse, lse_t)
        wa, wb = torch.exp(lse - mx), torch.exp(lse_t - mx)      # [H, S]
        oa, ob = o.view(S, H, D), o_t.view(S, H, D)
        waT, wbT = wa.t()[..., None], wb.t()[..., None]
        oa.copy_((waT * oa + wbT * ob) / (waT + wbT))
        lse.copy_(mx + torch.log(wa + wb))

    def finalize(self, o_acc, out):
        out.copy_(o_acc.view(out.shape))

    # "copy" transport: peers' blocks become readable after sync_peers; here
    # an all_gather stands in for the IPC mappings
    def share(self, shape, dtype, device, rank, world, group):
        self.world, self.group = world, group
        self.qkv = torch.empty(shape, dtype=torch.float64)
        return self.qkv

    def wait_released(self):
        pass

    def sync_peers(self):
        self.blocks = [torch.empty_like(self.qkv[1:3]) for _ in range(self.world)]
        dist.all_gather(self.blocks, self.qkv[1:3].contiguous(), group=self.group)

    def fetch(self, src_rank, slot, kv_recv):
        S = self.blocks[src_rank].shape[2]
        kv_recv[:, :, slot * S:(slot + 1) * S].copy_(self.blocks[src_rank])
        return src_rank

    def wait(self, token):
        pass

    def release(self):
        dist.barrier(group=self.group)


def _ring_worker(rank, world, port, S, H, D, q, k, v, result, transport):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        s_loc = S // world
        sl = slice(rank * s_loc, (rank + 1) * s_loc)
        ops = CpuRingOps(H, D, D ** -0.5)
        ring = RingAttention(ops, H, D, S, rank, world, "cpu", qkv_dtype=torch.float64,
                             transport=transport)
        out = torch.empty((1, s_loc, H * D), dtype=torch.float64)
        for _ in range(2):          # a second call reuses the buffers
            ring.forward(q[:, sl], k[:, sl], v[:, sl], out)
        result[rank] = out[0].numpy()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("transport", ["nccl", "copy"])
@pytest.mark.parametrize("world", [2, 4])
def test_ring_schedule_and_merge_gloo(world, transport):
    S, H, D = 48, 3, 16
    g = torch.Generator().manual_seed(world)
    q, k, v = (torch.randn((1, S, H, D), generator=g, dtype=torch.float64) for _ in range(3))
    mgr = mp.get_context("spawn").Manager()
    result = mgr.dict()
    mp.start_processes(_ring_worker, args=(world, _free_port(), S, H, D, q, k, v, result,
                                           transport),
                       nprocs=world, join=True, start_method="spawn")
    got = np.concatenate([result[r] for r in range(world)], 0)
    s = torch.einsum("shd,thd->hst", q[0], k[0]) * D ** -0.5
    want = torch.einsum("hst,thd->shd", torch.softmax(s, -1), v[0]).reshape(S, H * D)
    np.testing.assert_allclose(got, want.numpy(), rtol=0, atol=1e-12)
