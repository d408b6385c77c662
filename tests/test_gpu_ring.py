"""GPU: the sequence-sharded ring (dependencies of RingAttention).

test_ring_ops_emulated runs every virtual rank's steps in one process on one
GPU (shard prologue with global RoPE rows and global gain split, attention
with LSE merged in the kernel epilogue, final conversion) and checks each shard of O
against the oracle on the whole sequence. test_ring_multi_gpu runs the real
thing between processes (K/V blocks by NCCL P2P, or pulled from the owners'
exported buffers on the copy engines) and needs two GPUs; it is skipped on
one."""
import os
import socket

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _prep(S=2048, H=3):
    """First 2048 tokens of the Qwen-Edit case: 1024 text + 1024 image."""
    import llmr_attn as L
    from llmr_attn import configs as C
    return C.prepare(C.C5, L.rope_tables, seq_len=S, n_heads=H)


@pytest.mark.parametrize("P", [2, 4])
def test_ring_ops_emulated(ctx, P):
    import torch
    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.dist import RingOps
    from llmr_attn.runner import attn_config
    prep = _prep()
    _, S, H, D = prep.q.shape
    s_loc = S // P
    cfg = attn_config(C.C5, S)
    cfg.n_heads = H
    cfg.split_row = C.C5.split_row          # global split row: 1024 > S here
    dev = lambda a, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dt)
    qg, kg = dev(prep.q_gain, torch.float32), dev(prep.k_gain, torch.float32)
    cos, sin = dev(prep.cos, torch.float32), dev(prep.sin, torch.float32)
    # Use a split inside the sequence so shards straddle it.
    cfg.split_row = 300
    qkv = []
    for r in range(P):
        sl = slice(r * s_loc, (r + 1) * s_loc)
        ops = RingOps(ctx, cfg, s_loc, r * s_loc)
        buf = torch.empty((3, H, s_loc, D), dtype=torch.float16, device="cuda")
        ops.prologue(dev(prep.q[:, sl]), dev(prep.k[:, sl]), dev(prep.v[:, sl]), buf, qg, kg,
                     cos, sin)
        qkv.append((ops, buf))
    want = O.attention_block(prep.q[0], prep.k[0], prep.v[0], H, D, C.C5.scale, eps=C.C5.eps,
                             q_gain=prep.q_gain, k_gain=prep.k_gain, split_row=300,
                             cos=prep.cos, sin=prep.sin)
    for r in range(P):
        ops, buf = qkv[r]
        o_acc = torch.empty((s_loc, H * D), device="cuda")
        l_acc = torch.empty((H, s_loc), device="cuda")
        for t in range(P):
            src = qkv[(r - t) % P][1]
            ops.partial(buf[0], src[1], src[2], o_acc, l_acc, merge=t > 0)
        out = torch.empty((1, s_loc, H * D), device="cuda", dtype=torch.float32)
        ops.finalize(o_acc, out)
        ctx.sync()
        got = out[0].cpu().numpy()
        err = np.abs(got - want[r * s_loc:(r + 1) * s_loc])
        assert err.max() <= 2e-3 and err.mean() <= 2e-4, (r, err.max(), err.mean())


def _ring_worker(rank, world, port, result, transport):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "llm-runner_b200"), os.path.join(root, "oracle")]
    import torch
    import torch.distributed as dist
    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.dist import RingAttention, RingOps
    from llmr_attn.runner import attn_config
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        prep = _prep()
        _, S, H, D = prep.q.shape
        s_loc = S // world
        cfg = attn_config(C.C5, S)
        cfg.n_heads = H
        cfg.split_row = 300
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            ctx = L.Context(rank, stream=stream)
            dev = lambda a, dt=torch.bfloat16: torch.from_numpy(
                np.ascontiguousarray(a)).cuda().to(dt)
            sl = slice(rank * s_loc, (rank + 1) * s_loc)
            ring = RingAttention(RingOps(ctx, cfg, s_loc, rank * s_loc), H, D, S, rank, world,
                                 f"cuda:{rank}", transport=transport)
            out = torch.empty((1, s_loc, H * D), device="cuda", dtype=torch.float32)
            args = (dev(prep.q[:, sl]), dev(prep.k[:, sl]), dev(prep.v[:, sl]), out,
                    dev(prep.q_gain, torch.float32), dev(prep.k_gain, torch.float32),
                    dev(prep.cos, torch.float32), dev(prep.sin, torch.float32))
            for _ in range(3):      # later calls reuse the shared blocks
                ring.forward(*args)
            ctx.sync()
        result[rank] = out[0].cpu().numpy()
        torch.cuda.synchronize()
        dist.barrier()
        ring.close()
        ctx.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "copy"])
def test_ring_multi_gpu(transport):
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_ring_worker, args=(world, port, result, transport), nprocs=world,
                       join=True, start_method="spawn")
    prep = _prep()
    _, S, H, D = prep.q.shape
    from llmr_attn import configs as C
    want = O.attention_block(prep.q[0], prep.k[0], prep.v[0], H, D, C.C5.scale, eps=C.C5.eps,
                             q_gain=prep.q_gain, k_gain=prep.k_gain, split_row=300,
                             cos=prep.cos, sin=prep.sin)
    got = np.concatenate([result[r] for r in range(world)], 0)
    err = np.abs(got - want)
    assert err.max() <= 2e-3 and err.mean() <= 2e-4, (err.max(), err.mean())
