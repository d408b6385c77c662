"""GPU: the allocation-free entry point llmr_attention_fused_noalloc.

Some callers cannot allocate device memory: their HBM belongs to another
allocator (a serving runtime or host engine that reserves memory up front and
accounts for every byte), or they run latency-critical paths that must not
call cudaMalloc/cudaFree, which can synchronise the whole device. They call
this entry point, which uses a fixed scratch array inside the library instead
of a context workspace. The test calls it through the C ABI twice in a row
(different inputs each time, so stale scratch from the first call would show)
and compares each result with the regular entry point llmr_attention_fused:
bf16 input with norm + RoPE (the prologue writes the scratch), D = 64 and
128, fp16 input without norm / RoPE (read in place, no scratch), BHSD with
explicit strides, the LSE output, and fp16 / bf16 output. It also checks that
the calls after the first one allocate no device memory and that the status
query reports no expired wait.

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


def _noalloc(desc, q, k, v, o, qg=None, kg=None, cos=None, sin=None, lse=None):
    import torch
    import llmr_attn as L
    p = lambda t: None if t is None else t.data_ptr()
    return L.lib.llmr_attention_fused_noalloc(
        ctypes.byref(desc), p(q), p(k), p(v), p(qg), p(kg), p(cos), p(sin), p(o), p(lse),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream or None))


CASES = [
    # (D, in dtype, out dtype, layout, norm + RoPE, LSE)
    (64, "bf16", "f32", "bshd", True, False),
    (128, "f16", "f32", "bshd", False, True),      # direct: fp16 read in place, no scratch
    (64, "f16", "bf16", "bhsd", False, False),
    (128, "bf16", "f16", "bhsd", True, True),
]


@pytest.mark.parametrize("D,ind,outd,layout,normrope,use_lse", CASES)
def test_noalloc_variants_match_fused(D, ind, outd, layout, normrope, use_lse):
    import torch
    import llmr_attn as L
    from llmr_attn import configs as C
    torch.cuda.set_device(0)
    S, H = 517, 3
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
    code = {"bf16": L.BF16, "f16": L.F16, "f32": L.F32}
    bhsd = layout == "bhsd"
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, eps=1e-6, norm_q=normrope,
                       norm_k=normrope, rope=normrope, split_row=100 if normrope else 0,
                       layout=L.BHSD if bhsd else L.BSHD)
    cos = sin = None
    if normrope:
        ids = C.flux_ids(100, 21, 21)[:S]
        axes = (16, 24, 24) if D == 64 else (16, 56, 56)
        cos, sin = (torch.from_numpy(t).cuda() for t in L.rope_tables(ids, axes, 1e4))
    # BHSD with explicit strides: each head's rows padded to 8 extra elements.
    strides = None
    shape = (1, H, S, D) if bhsd else (1, S, H, D)
    if bhsd:
        rs = D + 8
        strides = {f"{t}_{n}": v for t in "qkv" for n, v in
                   (("row_stride", rs), ("head_stride", S * rs), ("batch_stride", H * S * rs))}
    ctx = L.Context(0)
    ctx.reserve(L.workspace_bytes(L.make_desc(cfg, 1, S, code[ind], code[outd],
                                              strides=strides)))
    free_after_first = None
    for call, seed in enumerate((11, 12, 13)):
        rng = np.random.default_rng(seed * 100 + D)
        def mk():
            a = C.round_to(rng.standard_normal(shape, dtype=np.float32), ind)
            if bhsd:
                pad = np.zeros((1, H, S, D + 8), np.float32)
                pad[..., :D] = a
                a = pad
            return torch.from_numpy(a).cuda().to(tdt[ind])
        q, k, v = mk(), mk(), mk()
        qg = torch.from_numpy(rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)).cuda()
        kg = torch.from_numpy(rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)).cuda()
        if not normrope:
            qg = kg = None
        want = torch.empty((1, S, H * D), device="cuda", dtype=tdt[outd])
        lse_w = torch.empty((1, H, S), device="cuda") if use_lse else None
        L.attention_fused(ctx, q, k, v, want, cfg, batch=1, seq_len=S, q_gain=qg, k_gain=kg,
                          cos=cos, sin=sin, lse=lse_w, strides=strides)
        ctx.sync()
        got = torch.full_like(want, float("nan"))
        lse_g = torch.full_like(lse_w, float("nan")) if use_lse else None
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        desc = L.make_desc(cfg, 1, S, code[ind], code[outd], lse=use_lse, strides=strides)
        rc = _noalloc(desc, q, k, v, got, qg, kg, cos, sin, lse_g)
        assert rc == L.OK, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info()[0]
        L.noalloc_status()  # raises on an expired device-side wait
        if call > 0:
            # Only the first call on a device may set anything up.
            assert free1 == free0, f"call {call}: device memory changed by {free0 - free1} B"
        else:
            free_after_first = free1
        assert torch.isfinite(got.float()).all(), f"call {call}: non-finite output"
        # The same kernels on the same operands: bit-identical to the fused op
        # (its parity with the oracle is covered by the parity tests).
        err = (got.float() - want.float()).abs()
        assert err.max().item() == 0.0, f"call {call}: max {err.max().item():.3e}"
        if use_lse:
            assert torch.equal(lse_g, lse_w), f"call {call}: LSE differs"
    assert free_after_first is not None
    ctx.close()
