"""GPU: the VAE mid-block attention (vae_attention, lib/shaders/diffusion.slang:
1828-1975; one head of D = 512 in dependencies/zimage.c3l/flux_vae.c3:493-538,
of D = 384 in dependencies/qwen_edit.c3l/qwen_vae.c3:430-464) on the wide-head
tensor-core kernel and on the exact fp32 path, against the oracle's
restatement of the shader (fp32, exact softmax over 4096-key tiles).

Tolerances: the tensor-core path rounds Q, K, V and P to fp16 (as the fused
op does for every head size): max abs <= 2e-3, mean abs <= 2e-4 on O. The
exact path computes in fp32: max abs <= 1e-5."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _t():
    import torch
    return torch


def _inputs(seed, S, C):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((S, C)).astype(np.float32) for _ in range(3)]


def _check(got, want, max_abs, mean_abs):
    err = np.abs(got.astype(np.float64) - want)
    assert err.max() <= max_abs and err.mean() <= mean_abs, (err.max(), err.mean())


@pytest.mark.parametrize("S,H,D", [
    (300, 1, 512),    # ragged last query tile and key block
    (129, 1, 384),    # Qwen VAE head size, one key past a block
    (5, 1, 512),      # fewer rows than one tile
    (640, 2, 384),    # two heads in [S, C]
    (4500, 1, 512),   # keys beyond the shader's first 4096-key tile
])
def test_vae_attention_mirror_vs_oracle(ctx, S, H, D):
    import llmr_attn as L
    torch = _t()
    q, k, v = _inputs(S * 7 + D, S, H * D)
    scale = D ** -0.5
    want = O.vae_attention(q, k, v, D, H, S, scale)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    o = torch.full((S, H * D), float("nan"), device="cuda")
    ctx.reserve(3 * S * H * D * 2)
    L.vae_attention(ctx, dq, dk, dv, o, D, H, S, scale)
    ctx.sync()
    _check(o.cpu().numpy(), want, 2e-3, 2e-4)


@pytest.mark.parametrize("S,D", [(300, 512), (129, 384)])
def test_vae_single_cta_kernel(ctx, monkeypatch, S, D):
    """The single-CTA wide kernel (LLMR_WIDE_SINGLE_CTA; the default is the
    CTA-pair kernel) on ragged cases."""
    import llmr_attn as L
    torch = _t()
    monkeypatch.setenv("LLMR_WIDE_SINGLE_CTA", "1")
    q, k, v = _inputs(S + D, S, D)
    want = O.vae_attention(q, k, v, D, 1, S, D ** -0.5)
    o = torch.empty((S, D), device="cuda")
    ctx.reserve(3 * S * D * 2)
    L.vae_attention(ctx, *(torch.from_numpy(a).cuda() for a in (q, k, v)), o, D, 1, S,
                    D ** -0.5)
    ctx.sync()
    _check(o.cpu().numpy(), want, 2e-3, 2e-4)


def test_vae_attention_channels_stride(ctx):
    """channels > n_heads * head_dim: rows of [S, C] with padding columns,
    which the op neither reads into the result nor writes."""
    import llmr_attn as L
    torch = _t()
    S, D, C = 200, 512, 576
    q, k, v = _inputs(3, S, C)
    want = O.vae_attention(q[:, :D], k[:, :D], v[:, :D], D, 1, S, D ** -0.5)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    o = torch.full((S, C), 7.0, device="cuda")
    ctx.reserve(3 * S * D * 2)
    L.vae_attention(ctx, dq, dk, dv, o, D, 1, S, D ** -0.5, channels=C)
    ctx.sync()
    got = o.cpu().numpy()
    _check(got[:, :D], want, 2e-3, 2e-4)
    assert np.all(got[:, D:] == 7.0)


def test_vae_attention_many_units_per_cta(ctx):
    """10240 queries: 40 tiles of 256 x 2 output parts = 80 units > 74 CTA
    pairs, so pairs walk more than one unit (Q reload, O hand-over between
    units). Checked on the first and last query tiles."""
    import llmr_attn as L
    torch = _t()
    S, D = 10240, 512
    q, k, v = _inputs(11, S, D)
    o = torch.empty((S, D), device="cuda")
    ctx.reserve(3 * S * D * 2)
    L.vae_attention(ctx, *(torch.from_numpy(a).cuda() for a in (q, k, v)), o, D, 1, S,
                    D ** -0.5)
    ctx.sync()
    got = o.cpu().numpy()
    for r0, r1 in ((0, 128), (S - 128, S)):
        want = O.vae_attention(q, k, v, D, 1, S, D ** -0.5, rows=(r0, r1))
        _check(got[r0:r1], want[r0:r1], 2e-3, 2e-4)


@pytest.mark.parametrize("D,S", [(512, 300), (384, 257)])
def test_vae_exact_path_vs_oracle(ctx, D, S):
    """LLMR_EXACT on a wide head: fp32 throughout, within 1e-5 of the shader."""
    import llmr_attn as L
    torch = _t()
    q, k, v = _inputs(D + S, S, D)
    scale = D ** -0.5
    want = O.vae_attention(q, k, v, D, 1, S, scale)
    cfg = L.AttnConfig(n_heads=1, head_dim=D, scale=scale, exact=True)
    ctx.reserve(L.workspace_bytes(L.make_desc(cfg, 1, S, L.F32, L.F32)))
    o = torch.empty((1, S, D), device="cuda")
    L.attention_fused(ctx, *(torch.from_numpy(a)[None].cuda() for a in (q, k, v)), o, cfg,
                      batch=1, seq_len=S)
    ctx.sync()
    _check(o[0].cpu().numpy(), want, 1e-5, 1e-6)


@pytest.mark.parametrize("in_dt,out_dt,layout", [
    ("f16", "bf16", "BHSD"),   # fp16 inputs are read in place (no workspace)
    ("bf16", "f16", "BSHD"),
    ("f32", "f32", "BHSD"),
])
def test_wide_fused_dtypes_layouts_lse(ctx, in_dt, out_dt, layout):
    """The fused op at D = 512 with batch 2 and 2 heads: input / output dtypes,
    both layouts, and the natural-log LSE against a float64 restatement."""
    import llmr_attn as L
    torch = _t()
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}
    B, H, S, D = 2, 2, 333, 512
    g = torch.Generator().manual_seed(5)
    shape = (B, S, H, D) if layout == "BSHD" else (B, H, S, D)
    qkv = [torch.randn(shape, generator=g).to(dt[in_dt]) for _ in range(3)]
    lay = L.BSHD if layout == "BSHD" else L.BHSD
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, layout=lay)
    ctx.reserve(L.workspace_bytes(L.make_desc(cfg, B, S, L._dtype_code(qkv[0]), L.F32)))
    o = torch.empty((B, S, H * D), device="cuda", dtype=dt[out_dt])
    lse = torch.empty((B, H, S), device="cuda")
    L.attention_fused(ctx, *(t.cuda() for t in qkv), o, cfg, batch=B, seq_len=S, lse=lse)
    ctx.sync()
    f = [t.float().numpy().astype(np.float64) for t in qkv]
    if layout == "BSHD":
        f = [a.transpose(0, 2, 1, 3) for a in f]        # -> [B, H, S, D]
    # fp16 operands, as the kernel rounds them
    r = [a.astype(np.float16).astype(np.float64) for a in f]
    s = np.einsum("bhqd,bhkd->bhqk", r[0], r[1]) * D ** -0.5
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m)
    want = np.einsum("bhqk,bhkd->bhqd", p / p.sum(-1, keepdims=True), r[2])
    want_lse = (m[..., 0] + np.log(p.sum(-1)))
    got = o.float().cpu().numpy().reshape(B, S, H, D).transpose(0, 2, 1, 3)
    tol = 2e-3 if out_dt == "f32" else 8e-3          # plus one 16-bit output rounding
    _check(got, want, tol, 2e-4 if out_dt == "f32" else 1e-3)
    assert np.abs(lse.cpu().numpy() - want_lse).max() <= 1e-3


@pytest.mark.parametrize("single", [False, True])
def test_wide_kv_len_differs_from_queries(ctx, monkeypatch, single):
    """kv_seq_len at D = 512: 200 queries over 333 keys (fp16 BHSD read in
    place), both wide kernels, against a float64 restatement."""
    import llmr_attn as L
    torch = _t()
    if single:
        monkeypatch.setenv("LLMR_WIDE_SINGLE_CTA", "1")
    rng = np.random.default_rng(9)
    S, T, D = 200, 333, 512
    q = rng.standard_normal((S, D)).astype(np.float16)
    k = rng.standard_normal((T, D)).astype(np.float16)
    v = rng.standard_normal((T, D)).astype(np.float16)
    cfg = L.AttnConfig(n_heads=1, head_dim=D, scale=D ** -0.5, layout=L.BHSD)
    o = torch.empty((1, S, D), device="cuda")
    L.attention_fused(ctx, *(torch.from_numpy(a)[None, None].cuda() for a in (q, k, v)), o, cfg,
                      batch=1, seq_len=S, kv_len=T)
    ctx.sync()
    s = q.astype(np.float64) @ k.astype(np.float64).T * D ** -0.5
    p = np.exp(s - s.max(-1, keepdims=True))
    want = (p / p.sum(-1, keepdims=True)) @ v.astype(np.float64)
    _check(o[0].cpu().numpy(), want, 2e-3, 2e-4)


def test_wide_rejects(ctx):
    import llmr_attn as L
    torch = _t()
    x = torch.zeros((1, 64, 1, 512), device="cuda", dtype=torch.float16)
    o = torch.empty((1, 64, 512), device="cuda")
    gain = torch.ones(512, device="cuda")
    cfg = L.AttnConfig(n_heads=1, head_dim=512, scale=0.04, norm_q=True)
    with pytest.raises(L.LlmrError) as ei:
        L.attention_fused(ctx, x, x, x, o, cfg, batch=1, seq_len=64, q_gain=gain)
    assert ei.value.status == L.EINVAL
    plain = L.AttnConfig(n_heads=1, head_dim=512, scale=0.04)
    with pytest.raises(L.LlmrError):
        L.attention_varlen(ctx, x, x, x, o, plain, [32, 32])
    odd = L.AttnConfig(n_heads=1, head_dim=256, scale=0.06)
    x2 = torch.zeros((1, 64, 1, 256), device="cuda", dtype=torch.float16)
    with pytest.raises(L.LlmrError):
        L.attention_fused(ctx, x2, x2, x2, o, odd, batch=1, seq_len=64)
