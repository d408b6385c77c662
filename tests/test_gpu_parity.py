"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and
the golden vectors. Tolerances are the north star's: on O, max-abs <= 2e-3 and
mean-abs <= 2e-4 for fp16/bf16 operands, <= 1e-5 for the fp32 config."""
import numpy as np
import pytest

import oracle as O
from conftest import load_golden

pytestmark = pytest.mark.gpu

TOL_MAX, TOL_MEAN = 2e-3, 2e-4


def _t():
    import torch
    return torch


def dev(a):
    return _t().from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    return t.float().cpu().numpy()


def check(got, want, tol_max=TOL_MAX, tol_mean=TOL_MEAN, what=""):
    assert got.shape == want.shape, (got.shape, want.shape)
    assert np.all(np.isfinite(got)), what + ": non-finite output"
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert err.max() <= tol_max and err.mean() <= tol_mean, \
        f"{what}: max {err.max():.3e} mean {err.mean():.3e}"


# ----------------------------------------------------------- reference op mirrors

def test_head_norm_mirror(ctx, manifest):
    import llmr_attn as L
    m = manifest["head_norm"]
    p = m["params"]
    x = dev(load_golden(m["x"]))
    L.batch_head_norm(ctx, x, dev(load_golden(m["gain"])), p["H"], p["D"], p["S"], p["eps"])
    ctx.sync()
    check(host(x), load_golden(m["out"]), 1e-5, 1e-6, "batch_head_norm")
    y = dev(load_golden(m["x"]))
    L.perhead_rmsnorm(ctx, y, dev(load_golden(m["gain"])), p["S"], p["H"], p["D"], p["eps"])
    ctx.sync()
    check(host(y), load_golden(m["out"]), 1e-5, 1e-6, "perhead_rmsnorm")


@pytest.mark.parametrize("direction", [0, 1])
def test_transpose_mirror(ctx, manifest, direction):
    import llmr_attn as L
    m = manifest["transpose"]
    p = m["params"]
    x = dev(load_golden(m["x"]))
    out = _t().empty_like(x)
    L.transpose_heads(ctx, x, out, p["S"], p["H"], p["D"], direction)
    ctx.sync()
    np.testing.assert_array_equal(host(out).reshape(-1),
                                  load_golden(m[f"out{direction}"]).reshape(-1))


def test_mrope_mirror(ctx, manifest):
    import llmr_attn as L
    m = manifest["mrope"]
    p = m["params"]
    x = dev(load_golden(m["x"]))
    L.mrope(ctx, x, dev(load_golden(m["cos"])), dev(load_golden(m["sin"])), p["S"], p["H"])
    ctx.sync()
    check(host(x), load_golden(m["out"]), 1e-6, 1e-7, "mrope")


def test_split_qkv_mirror(ctx, manifest):
    import llmr_attn as L
    m = manifest["split_qkv"]
    p = m["params"]
    qkv = dev(load_golden(m["qkv"]))
    q, k, v = (_t().empty((p["n_rows"], p["dim"]), device="cuda") for _ in range(3))
    L.split_qkv(ctx, qkv, q, k, v, p["dim"], p["n_rows"])
    ctx.sync()
    for name, t in (("q", q), ("k", k), ("v", v)):
        np.testing.assert_array_equal(host(t), load_golden(m[name]))


def test_flash_attention_v2_mirror(ctx, manifest):
    import llmr_attn as L
    m = manifest["fa2"]
    p = m["params"]
    ctx.reserve(3 * p["H"] * p["S"] * p["D"] * 2)
    o = _t().empty((p["S"], p["H"] * p["D"]), device="cuda")
    L.flash_attention_v2(ctx, dev(load_golden(m["q"])), dev(load_golden(m["k"])),
                         dev(load_golden(m["v"])), o, p["D"], p["H"], p["S"], p["scale"])
    ctx.sync()
    check(host(o), load_golden(m["out"]), what="flash_attention_v2")


def test_spatial_attention_mirror(ctx, manifest):
    import llmr_attn as L
    m = manifest["spatial"]
    p = m["params"]
    o = _t().empty((p["H"], p["S"], p["D"]), device="cuda")
    L.spatial_attention(ctx, dev(load_golden(m["q"])), dev(load_golden(m["k"])),
                        dev(load_golden(m["v"])), None, o, p["D"], p["H"], p["S"], p["scale"])
    ctx.sync()
    check(host(o), load_golden(m["out"]), 1e-5, 1e-5, "spatial_attention")


def test_fused_block_golden(ctx, manifest):
    """The fused op replaces the whole Flux block sequence of the fixture."""
    import llmr_attn as L
    m = manifest["block_flux"]
    p = m["params"]
    S, H, D = p["S"], p["H"], p["D"]
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=p["scale"], eps=p["eps"], norm_q=True,
                       norm_k=True, rope=True, split_row=p["split"])
    ctx.reserve(3 * S * H * D * 2)
    o = _t().empty((1, S, H * D), device="cuda")
    L.attention_fused(ctx, dev(load_golden(m["q"])), dev(load_golden(m["k"])),
                      dev(load_golden(m["v"])), o, cfg, batch=1, seq_len=S,
                      q_gain=dev(load_golden(m["q_gain"])), k_gain=dev(load_golden(m["k_gain"])),
                      cos=dev(load_golden(m["cos"])), sin=dev(load_golden(m["sin"])))
    ctx.sync()
    check(host(o)[0], load_golden(m["out"]), what="fused block")


# ------------------------------------------------------------- tensor-core kernel

def oracle_fa(q_bshd, k_bshd, v_bshd, scale, rows=None):
    """Reference flash_attention_v2 on BSHD inputs -> O [B,S,H*D]."""
    B, S, H, D = q_bshd.shape
    out = []
    for b in range(B):
        tr = lambda a: np.ascontiguousarray(a[b].transpose(1, 0, 2))
        qb = None if rows is None else (rows[0] // 16, (rows[1] + 15) // 16)
        out.append(O.flash_attention_v2(tr(q_bshd), tr(k_bshd), tr(v_bshd), D, H, S, scale,
                                        qb_range=qb))
    return np.stack(out)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [1, 15, 17, 33, 127, 128, 129, 255, 256, 257, 300, 1000])
def test_tc_kernel_ragged_shapes(ctx, D, S):
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(S * 7 + D)
    B, H = 2, 3
    q, k, v = (rng.standard_normal((B, S, H, D), dtype=np.float32) for _ in range(3))
    q, k, v = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
    scale = D ** -0.5
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=scale)
    o = torch.empty((B, S, H * D), device="cuda", dtype=torch.float32)
    L.attention_fused(ctx, dev(q).half(), dev(k).half(), dev(v).half(), o, cfg, batch=B,
                      seq_len=S)
    ctx.sync()
    check(host(o), oracle_fa(q, k, v, scale).reshape(B, S, H * D), what=f"S={S} D={D}")


@pytest.mark.parametrize("D", [64, 128])
def test_tc_kernel_many_units_per_cta(ctx, D):
    """More (b, h, 256-query) units than SMs: the persistent kernel walks
    several units per CTA (TMEM, barriers and the K/V ring carry over), with
    a ragged last tile and a ragged last key block in every unit."""
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(300 + D)
    B, S, H = 3, 257, 52          # 3 * 52 * 2 = 312 units
    q, k, v = (rng.standard_normal((B, S, H, D), dtype=np.float32) for _ in range(3))
    q, k, v = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
    scale = D ** -0.5
    o = torch.empty((B, S, H * D), device="cuda", dtype=torch.float32)
    L.attention_fused(ctx, dev(q).half(), dev(k).half(), dev(v).half(), o,
                      L.AttnConfig(n_heads=H, head_dim=D, scale=scale), batch=B, seq_len=S)
    ctx.sync()
    check(host(o), oracle_fa(q, k, v, scale).reshape(B, S, H * D), what=f"units D={D}")


@pytest.mark.parametrize("D", [64, 128])
def test_tc_kernel_rescale_paths(ctx, D):
    """Scores that jump inside later key blocks, at different 32-key chunk
    positions: some jumps stay below the lazy-rescale threshold (P up to
    2^12.7 against the stale max), the others pass 2^15 and force O and l to
    be rescaled before P is written."""
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(21 + D)
    B, S, H = 1, 900, 2
    q = rng.standard_normal((B, S, H, D), dtype=np.float32) * 0.2
    k = rng.standard_normal((B, S, H, D), dtype=np.float32) * 0.2
    v = rng.standard_normal((B, S, H, D), dtype=np.float32)
    q[..., 0] += 2.0                     # every query shares a component on dim 0
    # (key position, size): block 1 chunk 0, block 2 chunk 1, block 3 chunk 3,
    # block 4 chunk 2, block 6 chunk 0; in log2(P) the jumps are about
    # +12.7 (no rescale), then +23, +38 and +76 (each a rescale) for D=128.
    for pos, size in ((150, 10.0), (2 * 128 + 40, 60.0), (3 * 128 + 100, 150.0),
                      (4 * 128 + 70, 300.0), (6 * 128 + 5, 600.0)):
        k[0, pos, :, :] = 0.0
        k[0, pos, :, 0] = size
    q, k, v = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
    scale = D ** -0.5
    o = torch.empty((B, S, H * D), device="cuda", dtype=torch.float32)
    L.attention_fused(ctx, dev(q).half(), dev(k).half(), dev(v).half(), o,
                      L.AttnConfig(n_heads=H, head_dim=D, scale=scale), batch=B, seq_len=S)
    ctx.sync()
    check(host(o), oracle_fa(q, k, v, scale).reshape(B, S, H * D), what=f"rescale D={D}")


@pytest.mark.parametrize("in_dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("out_dt", ["f32", "f16", "bf16"])
def test_tc_kernel_dtypes(ctx, in_dt, out_dt):
    import llmr_attn as L
    from llmr_attn.configs import round_to
    from llmr_attn.runner import torch_dtype
    torch = _t()
    rng = np.random.default_rng(3)
    B, S, H, D = 1, 333, 2, 128
    q, k, v = (round_to(rng.standard_normal((B, S, H, D), dtype=np.float32), in_dt)
               for _ in range(3))
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5)
    ctx.reserve(3 * B * S * H * D * 2)
    o = torch.empty((B, S, H * D), device="cuda", dtype=torch_dtype(out_dt))
    td = torch_dtype(in_dt)
    L.attention_fused(ctx, dev(q).to(td), dev(k).to(td), dev(v).to(td), o, cfg, batch=B,
                      seq_len=S)
    ctx.sync()
    want = oracle_fa(q, k, v, D ** -0.5).reshape(B, S, H * D)
    want = round_to(want, out_dt)
    # fp16/bf16 output adds one output rounding (<= 2^-9 relative for bf16).
    tmax = TOL_MAX if out_dt != "bf16" else 2e-3 + 4e-3
    check(host(o), want, tmax, 1e-3 if out_dt == "bf16" else TOL_MEAN, f"{in_dt}->{out_dt}")


def test_tc_kernel_bhsd_and_fused_qkv_strides(ctx):
    """BHSD layout, and a fused QKV buffer [S, 3*H*D] addressed by strides
    (replaces split_qkv, depth.slang:40-58)."""
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(4)
    B, S, H, D = 1, 200, 4, 64
    qkv = rng.standard_normal((B, S, 3, H, D), dtype=np.float32).astype(np.float16)
    qkv_d = torch.from_numpy(qkv).cuda()
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=0.125)
    o = torch.empty((B, S, H * D), device="cuda")
    st = {"q_row_stride": 3 * H * D, "k_row_stride": 3 * H * D, "v_row_stride": 3 * H * D,
          "q_batch_stride": S * 3 * H * D, "k_batch_stride": S * 3 * H * D,
          "v_batch_stride": S * 3 * H * D}
    flat = qkv_d.view(-1)
    L.attention_fused(ctx, flat[0:], flat[H * D:], flat[2 * H * D:], o, cfg, batch=B,
                      seq_len=S, strides=st)
    ctx.sync()
    q, k, v = (qkv[:, :, i].astype(np.float32) for i in range(3))
    want = oracle_fa(q, k, v, 0.125).reshape(B, S, H * D)
    check(host(o), want, what="fused-qkv strides")
    # BHSD input
    qh, kh, vh = (torch.from_numpy(np.ascontiguousarray(a.transpose(0, 2, 1, 3))).cuda().half()
                  for a in (q, k, v))
    cfg2 = L.AttnConfig(n_heads=H, head_dim=D, scale=0.125, layout=L.BHSD)
    o2 = torch.empty_like(o)
    L.attention_fused(ctx, qh, kh, vh, o2, cfg2, batch=B, seq_len=S)
    ctx.sync()
    check(host(o2), want, what="bhsd")


def test_fused_norm_rope_vs_oracle(ctx):
    """Norm with a txt/img gain split, RoPE from host tables, bf16 inputs."""
    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.runner import to_device
    prep = C.prepare(C.C3, L.rope_tables, seq_len=700, n_heads=3)
    dc = to_device(prep)
    ctx.reserve(L.workspace_bytes(dc.desc()))
    dc.run(ctx)
    ctx.sync()
    want = O.attention_block(prep.q[0], prep.k[0], prep.v[0], 3, 128, C.C3.scale, eps=C.C3.eps,
                             q_gain=prep.q_gain, k_gain=prep.k_gain, split_row=512,
                             cos=prep.cos, sin=prep.sin)
    check(host(dc.o)[0], C.round_to(want, "bf16"), TOL_MAX + 4e-3, 1e-3, "fused norm+rope")
    # the same call with an fp32 output is held to the plain tolerance
    dc.o = _t().empty(dc.o.shape, device="cuda", dtype=_t().float32)
    dc.run(ctx)
    ctx.sync()
    check(host(dc.o)[0], want, what="fused norm+rope f32 out")


def test_lse_output(ctx):
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(8)
    B, S, H, D = 1, 390, 2, 128
    q, k, v = (rng.standard_normal((B, S, H, D), dtype=np.float32).astype(np.float16)
               .astype(np.float32) for _ in range(3))
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5)
    o = torch.empty((B, S, H * D), device="cuda")
    lse = torch.empty((B, H, S), device="cuda")
    L.attention_fused(ctx, dev(q).half(), dev(k).half(), dev(v).half(), o, cfg, batch=B,
                      seq_len=S, lse=lse)
    ctx.sync()
    s = np.einsum("shd,thd->hst", q[0].astype(np.float64), k[0].astype(np.float64)) * D ** -0.5
    mx = s.max(-1, keepdims=True)
    want = (mx + np.log(np.exp(s - mx).sum(-1, keepdims=True)))[..., 0]
    assert np.abs(host(lse)[0] - want).max() < 1e-3


@pytest.mark.parametrize("D", [64, 128])
def test_merge_flag_combines_key_blocks(ctx, D):
    """LLMR_MERGE: attention over key block A, then over key block B merged
    into the same fp32 O / LSE, equals attention over the keys of A and B
    together (as the ring does with one block per step). Block B has a much
    larger logit range, so the merge weights are far from 1/2; S is not a
    tile multiple."""
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(D)
    S, H = 333, 2
    q = rng.standard_normal((S, H, D)).astype(np.float16).astype(np.float32)
    k = rng.standard_normal((2, S, H, D)).astype(np.float16).astype(np.float32)
    k[1] = (k[1] * 3.0).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((2, S, H, D)).astype(np.float16).astype(np.float32)
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, layout=L.BHSD)

    def bhsd(x):
        return dev(x.transpose(1, 0, 2)).half().contiguous()

    qh = bhsd(q)
    o = torch.empty((S, H * D), device="cuda")
    lse = torch.empty((H, S), device="cuda")
    for i in range(2):
        L.attention_fused(ctx, qh, bhsd(k[i]), bhsd(v[i]), o, cfg, batch=1, seq_len=S,
                          lse=lse, merge=i > 0)
    ctx.sync()
    kk = np.concatenate([k[0], k[1]], 0).astype(np.float64)
    vv = np.concatenate([v[0], v[1]], 0).astype(np.float64)
    s = np.einsum("shd,thd->hst", q.astype(np.float64), kk) * D ** -0.5
    mx = s.max(-1, keepdims=True)
    p = np.exp(s - mx)
    want_lse = (mx + np.log(p.sum(-1, keepdims=True)))[..., 0]
    want = np.einsum("hst,thd->shd", p / p.sum(-1, keepdims=True), vv).reshape(S, H * D)
    check(host(o), want, what=f"merge D={D}")
    assert np.abs(host(lse) - want_lse).max() < 1e-3
    # misuse: merge into a non-fp32 output, or without LSE, is rejected
    o16 = torch.empty((S, H * D), device="cuda", dtype=torch.float16)
    kh = bhsd(k[0])
    with pytest.raises(L.LlmrError) as ei:
        L.attention_fused(ctx, qh, kh, kh, o16, cfg, batch=1, seq_len=S, lse=lse, merge=True)
    assert ei.value.status == L.EINVAL
    with pytest.raises(L.LlmrError) as ei:
        L.attention_fused(ctx, qh, kh, kh, o, cfg, batch=1, seq_len=S, merge=True)
    assert ei.value.status == L.EINVAL


@pytest.mark.parametrize("D", [64, 128])
def test_kv_len_differs_from_queries(ctx, D):
    """kv_seq_len: 300 queries over two key blocks of 130 and 611 keys (both
    ragged), the second merged into the first; the K/V of each block are
    strided views into one buffer of all 741 keys, as the ring's received
    blocks are. Equals attention over all 741 keys."""
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(40 + D)
    S, T1, T2, H = 300, 130, 611, 3
    T = T1 + T2
    q = rng.standard_normal((S, H, D)).astype(np.float16).astype(np.float32)
    k = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, layout=L.BHSD)
    qh = dev(q.transpose(1, 0, 2)).half().contiguous()          # [H, S, D]
    kh = dev(k.transpose(1, 0, 2)).half().contiguous()          # [H, T, D]
    vh = dev(v.transpose(1, 0, 2)).half().contiguous()
    o = torch.empty((S, H * D), device="cuda")
    lse = torch.empty((H, S), device="cuda")
    for i, (a, n) in enumerate(((0, T1), (T1, T2))):
        st = {"k_row_stride": D, "v_row_stride": D, "k_head_stride": T * D,
              "v_head_stride": T * D}
        L.attention_fused(ctx, qh, kh[:, a:a + n], vh[:, a:a + n], o, cfg, batch=1, seq_len=S,
                          lse=lse, merge=i > 0, kv_len=n, strides=st)
    ctx.sync()
    s = np.einsum("shd,thd->hst", q.astype(np.float64), k.astype(np.float64)) * D ** -0.5
    mx = s.max(-1, keepdims=True)
    p = np.exp(s - mx)
    want = np.einsum("hst,thd->shd", p / p.sum(-1, keepdims=True),
                     v.astype(np.float64)).reshape(S, H * D)
    check(host(o), want, what=f"kv_len D={D}")
    want_lse = (mx + np.log(p.sum(-1, keepdims=True)))[..., 0]
    assert np.abs(host(lse) - want_lse).max() < 1e-3
    # a different key count with a prologue (norm) is rejected
    bad = L.AttnConfig(n_heads=H, head_dim=D, scale=0.1, layout=L.BHSD, norm_q=True)
    g = torch.ones(D, device="cuda")
    ctx.reserve(3 * H * S * D * 2)
    with pytest.raises(L.LlmrError) as ei:
        L.attention_fused(ctx, qh, kh, vh, o, bad, batch=1, seq_len=S, q_gain=g, kv_len=T)
    assert ei.value.status == L.EINVAL


# ----------------------------------------------------------------- configurations

def _run_case(ctx, case, rows_windows=None, **over):
    """Runs a configuration with an fp32 output (so the strict tolerance
    applies to the arithmetic) and compares windows of rows with the oracle."""
    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.runner import to_device
    prep = C.prepare(case, L.rope_tables, **over)
    dc = to_device(prep, out_dtype="f32")
    ctx.reserve(L.workspace_bytes(dc.desc()))
    dc.run(ctx)
    ctx.sync()
    got = host(dc.o)
    B, S, H, D = prep.q.shape
    split = min(case.split_row, S)
    for b in range(B):
        for (r0, r1) in (rows_windows or [(0, S)]):
            want = O.attention_block(prep.q[b], prep.k[b], prep.v[b], H, D, case.scale,
                                     eps=case.eps, q_gain=prep.q_gain, k_gain=prep.k_gain,
                                     split_row=split, cos=prep.cos, sin=prep.sin,
                                     exact=case.exact, rows=(r0, r1))
            check(got[b, r0:r1], want[r0:r1], case.tol_max, case.tol_mean,
                  f"{case.name} b={b} rows {r0}:{r1}")
    return dc, prep, got


def test_config_plumbing_fp32_exact(ctx):
    from llmr_attn import configs as C
    _run_case(ctx, C.C1)


def test_config_depth_fp16(ctx):
    from llmr_attn import configs as C
    _run_case(ctx, C.C2)


def test_config_flux_bf16_full(ctx):
    from llmr_attn import configs as C
    from llmr_attn.configs import round_to
    dc, prep, got = _run_case(ctx, C.C3)
    # The bf16 output of the same call is the RNE rounding of the fp32 one.
    dc.o = _t().empty(dc.o.shape, device="cuda", dtype=_t().bfloat16)
    dc.run(ctx)
    ctx.sync()
    np.testing.assert_array_equal(host(dc.o), round_to(got, "bf16"))


def test_config_zimage_cfg_full(ctx):
    """Z-Image CFG (B2 H30 S4352): every row of both batch elements against
    the oracle."""
    from llmr_attn import configs as C
    _run_case(ctx, C.C4)


def _f64_block(prep, case, b, chunk=1024):
    """fp64 restatement, on the GPU, of the oracle's block for batch element
    b, every row: per-head RMSNorm x / sqrt(mean(x^2) + eps) * g with the
    gain set chosen by the row's side of split_row, the interleaved RoPE
    rotation from the tables, Q / K / V rounded to fp16 (the rounding the
    reference applies on load), exact softmax attention. [S, H*D] fp64."""
    torch = _t()
    q, k, v = (torch.from_numpy(np.ascontiguousarray(a[b])).cuda().double()
               for a in (prep.q, prep.k, prep.v))
    S, H, D = q.shape
    split = min(case.split_row, S)

    def norm(x, g):
        if g is None:
            return x
        g = torch.from_numpy(np.asarray(g, np.float32).reshape(-1, D)).cuda().double()
        sel = torch.zeros(S, dtype=torch.long, device="cuda")
        if g.shape[0] > 1 and split > 0:
            sel[split:] = 1
        r = torch.rsqrt((x * x).mean(-1, keepdim=True) + case.eps)
        return x * r * g[sel][:, None, :]

    def rope(x):
        if prep.cos is None:
            return x
        c = torch.from_numpy(prep.cos[:S]).cuda().double()[:, None, :]
        s_ = torch.from_numpy(prep.sin[:S]).cuda().double()[:, None, :]
        out = torch.empty_like(x)
        out[..., 0::2] = x[..., 0::2] * c - x[..., 1::2] * s_
        out[..., 1::2] = x[..., 0::2] * s_ + x[..., 1::2] * c
        return out

    qn = rope(norm(q, prep.q_gain)).half().double()
    kn = rope(norm(k, prep.k_gain)).half().double()
    vn = v.half().double()
    out = torch.empty((S, H, D), dtype=torch.float64, device="cuda")
    for h in range(H):
        for r0 in range(0, S, chunk):
            sc = (qn[r0:r0 + chunk, h] @ kn[:, h].T) * case.scale
            out[r0:r0 + chunk, h] = torch.softmax(sc, dim=-1) @ vn[:, h]
    return out.reshape(S, H * D)


def test_config_qwen_long(ctx):
    """Qwen-Edit (B1 H24 S33792): row windows against the oracle (its full
    output would take minutes of CPU), and every row of every head against an
    fp64 restatement of the same block on the GPU."""
    from llmr_attn import configs as C
    S = C.C5.seq_len
    dc, prep, _ = _run_case(ctx, C.C5, rows_windows=[(1008, 1072), (S - 32, S)])
    want = _f64_block(prep, C.C5, 0)
    err = (dc.o[0].double() - want).abs()
    assert bool(torch_all_finite(dc.o))
    emax, emean = err.max().item(), err.mean().item()
    assert emax <= TOL_MAX and emean <= TOL_MEAN, f"qwen full: max {emax:.3e} mean {emean:.3e}"


def torch_all_finite(t):
    return _t().isfinite(t).all()


# ------------------------------------------------------------------ error behaviour

def test_errors_are_reported(ctx):
    import llmr_attn as L
    torch = _t()
    x = torch.zeros((1, 16, 2, 96), device="cuda", dtype=torch.float16)
    o = torch.zeros((1, 16, 192), device="cuda", dtype=torch.float16)
    with pytest.raises(L.LlmrError) as ei:
        L.attention_fused(ctx, x, x, x, o, L.AttnConfig(n_heads=2, head_dim=96, scale=0.1),
                          batch=1, seq_len=16)
    assert ei.value.status == L.EINVAL and "head_dim" in str(ei.value)
    big = torch.zeros((1, 16, 2, 128), device="cuda", dtype=torch.bfloat16)
    ob = torch.zeros((1, 16, 256), device="cuda", dtype=torch.bfloat16)
    tiny = L.Context(0, workspace_bytes=64)
    with pytest.raises(L.LlmrError) as ei:
        L.attention_fused(tiny, big, big, big, ob, L.AttnConfig(n_heads=2, head_dim=128,
                                                                scale=0.1),
                          batch=1, seq_len=16)
    assert ei.value.status == L.ENOMEM
    tiny.close()
    with pytest.raises(L.LlmrError):
        L.attention_fused(ctx, big, big, big, ob, L.AttnConfig(n_heads=2, head_dim=128,
                                                               scale=-1.0), batch=1, seq_len=16)
    ctx.sync()


def test_bounded_wait_timeout_is_reported(ctx):
    """A device-side wait that can never complete gives up after its limit;
    the context reports LLMR_ETIMEOUT at sync and stays usable (failure
    detection without a GPU fault or hang)."""
    import llmr_attn as L
    torch = _t()
    ctx.sync()
    ctx.check(L.lib.llmr_selftest_wait_timeout(ctx.handle, 20_000_000))  # 20 ms
    with pytest.raises(L.LlmrError) as ei:
        ctx.sync()
    assert ei.value.status == L.ETIMEOUT
    ctx.sync()  # the error word was cleared
    # the context still runs the op correctly
    rng = np.random.default_rng(9)
    q = rng.standard_normal((1, 100, 2, 64), dtype=np.float32).astype(np.float16).astype(np.float32)
    o = torch.empty((1, 100, 128), device="cuda")
    L.attention_fused(ctx, dev(q).half(), dev(q).half(), dev(q).half(), o,
                      L.AttnConfig(n_heads=2, head_dim=64, scale=0.125), batch=1, seq_len=100)
    ctx.sync()
    check(host(o), oracle_fa(q, q, q, 0.125).reshape(1, 100, 128), what="after timeout")
    with pytest.raises(L.LlmrError):
        ctx.check(L.lib.llmr_selftest_wait_timeout(ctx.handle, 0))


# -------------------------------------------------------------- variable length

@pytest.mark.parametrize("D,lens", [(128, (300, 129, 1000)), (64, (17, 640)),
                                    (128, (4352, 4096))])
def test_varlen_packed_sequences(ctx, D, lens):
    """llmr_attention_varlen: packed sequences of different lengths (the CFG
    pair with different text lengths is the last case) each equal the
    oracle's block on that sequence alone, with QK-RMSNorm and per-sequence
    RoPE tables concatenated in packing order."""
    import llmr_attn as L
    torch = _t()
    rng = np.random.default_rng(sum(lens) + D)
    H, T = 3, sum(lens)
    q, k, v = (rng.standard_normal((T, H, D), dtype=np.float32) for _ in range(3))
    q, k, v = (a.astype(np.float16).astype(np.float32) for a in (q, k, v))
    gq = rng.uniform(0.8, 1.2, D).astype(np.float32)
    gk = rng.uniform(0.8, 1.2, D).astype(np.float32)
    axes = (16, 56, 56) if D == 128 else (16, 24, 24)
    tables = []
    for i, n in enumerate(lens):   # each sequence has its own position ids
        pos = np.stack([np.full(n, i), np.arange(n) // 32, np.arange(n) % 32], 1).astype(np.int32)
        tables.append(L.rope_tables(pos, axes, 10000.0))
    cos = np.concatenate([c for c, _ in tables]); sin = np.concatenate([s for _, s in tables])
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, norm_q=True, norm_k=True,
                       rope=True, eps=1e-6)
    ctx.reserve(3 * T * H * D * 2)
    o = torch.empty((1, T, H * D), device="cuda")
    L.attention_varlen(ctx, dev(q).half(), dev(k).half(), dev(v).half(), o, cfg, lens,
                       q_gain=dev(gq), k_gain=dev(gk), cos=dev(cos), sin=dev(sin))
    ctx.sync()
    got = host(o)[0]
    off = 0
    for i, n in enumerate(lens):
        sl = slice(off, off + n)
        rows = (0, n) if n <= 1024 else (n - 300, n)     # long sequence: its last rows
        want = O.attention_block(q[sl].reshape(n, -1), k[sl].reshape(n, -1),
                                 v[sl].reshape(n, -1), H, D, D ** -0.5, eps=1e-6,
                                 q_gain=gq, k_gain=gk, cos=tables[i][0], sin=tables[i][1],
                                 rows=rows)
        check(got[sl][rows[0]:rows[1]], want[rows[0]:rows[1]], what=f"seq {i} len {n}")
        off += n


def test_varlen_rejects(ctx):
    import llmr_attn as L
    torch = _t()
    x = torch.zeros((1, 64, 2, 128), device="cuda", dtype=torch.float16)
    o = torch.empty((1, 64, 256), device="cuda")
    cfg = L.AttnConfig(n_heads=2, head_dim=128, scale=0.1)
    with pytest.raises(L.LlmrError) as ei:
        L.attention_varlen(ctx, x, x, x, o, cfg, (30, 30))      # lengths do not sum
    assert ei.value.status == L.EINVAL
    with pytest.raises(L.LlmrError) as ei:
        L.attention_varlen(ctx, x, x, x, o, L.AttnConfig(n_heads=2, head_dim=128, scale=0.1,
                                                         split_row=8), (32, 32))
    assert ei.value.status == L.EINVAL


def test_fused_two_devices_one_process():
    """One process driving two GPUs (a context per device, calls alternating
    between them): kernel attributes are per device, so each device must get
    its own set-up. Every result is checked against the oracle."""
    torch = _t()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import llmr_attn as L
    from llmr_attn import configs as C
    from llmr_attn.runner import to_device
    prep = C.prepare(C.C3, L.rope_tables, seq_len=384, n_heads=2)
    want = O.attention_block(prep.q[0], prep.k[0], prep.v[0], 2, 128, C.C3.scale,
                             eps=C.C3.eps, q_gain=prep.q_gain, k_gain=prep.k_gain,
                             split_row=min(C.C3.split_row, 384), cos=prep.cos, sin=prep.sin)
    ctxs, cases = [], []
    for d in (0, 1):
        torch.cuda.set_device(d)
        dc = to_device(prep, device=d, out_dtype="f32")
        c = L.Context(d)
        c.reserve(L.workspace_bytes(dc.desc()))
        ctxs.append(c)
        cases.append(dc)
    for _ in range(2):
        for d in (1, 0):  # device 1 first: a per-process flag would skip its set-up
            cases[d].o.fill_(float("nan"))
            cases[d].run(ctxs[d])
            ctxs[d].sync()
            check(host(cases[d].o)[0], want, what=f"cuda:{d}")
    for c in ctxs:
        c.close()
    torch.cuda.set_device(0)
