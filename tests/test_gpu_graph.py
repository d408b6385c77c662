"""GPU: the fused op captured into a CUDA graph and replayed gives the eager
call's output bit for bit, also after new inputs are copied into the captured
buffers; the capture holds the library's two launches (prologue, attention
with programmatic dependent launch). This is how a serving loop replaces the
reference's recorded command buffer (lib/vulkan/graph.c3: the RenderGraph is
recorded once and submitted per step)."""
import numpy as np
import pytest
import torch

import llmr_attn as L
from llmr_attn import configs as C
from llmr_attn.runner import to_device

pytestmark = pytest.mark.gpu


def _case(seq_len, n_heads, seed):
    prep = C.prepare(C.C3, L.rope_tables, seq_len=seq_len, n_heads=n_heads)
    rng = np.random.default_rng(seed)
    prep.q = C.round_to(rng.standard_normal(prep.q.shape, dtype=np.float32), "bf16")
    return prep


@pytest.mark.parametrize("out_dtype", ["bf16", "f32"])
def test_fused_op_replays_from_a_cuda_graph(out_dtype):
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ctx = L.Context(0, stream=s)
        dc = to_device(_case(1000, 4, 1), out_dtype=out_dtype)
        other = to_device(_case(1000, 4, 2), out_dtype=out_dtype)
        ctx.reserve(L.workspace_bytes(dc.desc()))
        # Eager references for both input sets.
        other.run(ctx)
        dc.run(ctx)
        ctx.sync()
        ref_a = dc.o.clone()
        ref_b = other.o.clone()
        dc.o.fill_(float("nan"))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    n0 = ctx.launches
    with torch.cuda.graph(g, stream=s):
        dc.run(ctx)
    assert ctx.launches - n0 == 2  # prologue + attention, recorded once
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ctx.sync()
    assert torch.equal(dc.o, ref_a)
    # New inputs into the captured buffers: the replay computes them.
    with torch.cuda.stream(s):
        dc.q.copy_(other.q)
        dc.o.fill_(float("nan"))
        g.replay()
    torch.cuda.synchronize()
    ctx.sync()
    assert torch.equal(dc.o, ref_b)
    del g
    ctx.close()
