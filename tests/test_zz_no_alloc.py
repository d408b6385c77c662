"""GPU: the allocation-free entry point llmr_attention_fused_noalloc.

Some callers cannot allocate device memory: their HBM belongs to another
allocator (a serving runtime or host engine that reserves memory up front and
accounts for every byte), or they run latency-critical paths that must not
call cudaMalloc/cudaFree, which can synchronise the whole device. They call
this entry point, which uses a fixed scratch array inside the library instead
of a context workspace. The test calls it through the C ABI twice in a row
(different inputs each time, so stale scratch from the first call would show)
and compares each result with the regular entry point llmr_attention_fused.

This file is named so that pytest collects it last; it creates everything it
uses, so it also passes when run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_MAX, TOL_MEAN = 2e-3, 2e-4


def _inputs(seed, S, H, D):
    import torch
    from llmr_attn import configs as C
    rng = np.random.default_rng(seed)
    q, k, v = (C.round_to(rng.standard_normal((1, S, H, D), dtype=np.float32), "bf16")
               for _ in range(3))
    qg = rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)
    kg = rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)
    dev = lambda a, dt=torch.bfloat16: torch.from_numpy(a).cuda().to(dt)
    return (dev(q), dev(k), dev(v), dev(qg, torch.float32), dev(kg, torch.float32))


@pytest.mark.parametrize("S,H", [(700, 3), (1370, 2)])
def test_noalloc_matches_fused_two_calls(S, H):
    import torch
    import llmr_attn as L
    from llmr_attn import configs as C
    torch.cuda.set_device(0)
    D = 128
    ids = C.flux_ids(512, 64, 64)[:S]
    cos, sin = (torch.from_numpy(t).cuda() for t in L.rope_tables(ids, (16, 56, 56), 1e4))
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, eps=1e-6, norm_q=True,
                       norm_k=True, rope=True, split_row=512)
    ctx = L.Context(0)
    ctx.reserve(L.workspace_bytes(L.make_desc(cfg, 1, S, L.BF16, L.F32)))
    for call, seed in enumerate((101, 202)):
        q, k, v, qg, kg = _inputs(seed + S, S, H, D)
        want = torch.empty((1, S, H * D), device="cuda", dtype=torch.float32)
        L.attention_fused(ctx, q, k, v, want, cfg, batch=1, seq_len=S, q_gain=qg, k_gain=kg,
                          cos=cos, sin=sin)
        ctx.sync()
        got = torch.full((1, S, H * D), float("nan"), device="cuda", dtype=torch.float32)
        desc = L.make_desc(cfg, 1, S, L.BF16, L.F32)
        rc = L.lib.llmr_attention_fused_noalloc(
            ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), qg.data_ptr(),
            kg.data_ptr(), cos.data_ptr(), sin.data_ptr(), got.data_ptr(), None,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream or None))
        assert rc == L.OK, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        err = (got - want).abs()
        assert torch.isfinite(got).all(), f"call {call}: non-finite output"
        assert err.max().item() <= TOL_MAX and err.mean().item() <= TOL_MEAN, \
            f"call {call}: max {err.max().item():.3e} mean {err.mean().item():.3e}"
    ctx.close()


def test_noalloc_rejects_oversize_and_exact():
    import torch
    import llmr_attn as L
    torch.cuda.set_device(0)
    x = torch.zeros(1024, device="cuda", dtype=torch.bfloat16)
    o = torch.zeros(1024, device="cuda", dtype=torch.bfloat16)
    # 3 * B*H*S*D * 2 bytes of scratch > the fixed maximum: refused before any launch.
    big = L.AttnConfig(n_heads=24, head_dim=128, scale=0.088, norm_q=True, norm_k=True)
    desc = L.make_desc(big, 1, 16384, L.BF16, L.BF16)
    assert 3 * 24 * 16384 * 128 * 2 > L.NOALLOC_SCRATCH_BYTES
    rc = L.lib.llmr_attention_fused_noalloc(ctypes.byref(desc), x.data_ptr(), x.data_ptr(),
                                            x.data_ptr(), x.data_ptr(), x.data_ptr(), None,
                                            None, o.data_ptr(), None, None)
    assert rc == L.ENOMEM
    ex = L.AttnConfig(n_heads=1, head_dim=64, scale=0.125, exact=True)
    rc = L.lib.llmr_attention_fused_noalloc(ctypes.byref(L.make_desc(ex, 1, 8, L.F32, L.F32)),
                                            x.data_ptr(), x.data_ptr(), x.data_ptr(), None,
                                            None, None, None, o.data_ptr(), None, None)
    assert rc == L.EINVAL
