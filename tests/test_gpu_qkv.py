"""GPU: the QKV projection with the attention prologue in its epilogue
(llmr_qkv_project) against a float64 GEMM of the same fp16/bf16 operands
followed by the oracle's batch_head_norm and mrope (the reference's
batch_matmul_f16_coopmat -> batch_head_norm -> mrope sequence,
dependencies/zimage.c3l/dit.c3:1437-1450), and end to end through the
attention kernel."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _t():
    import torch
    return torch


def _inputs(seed, B, S, hidden, H, D, dtype):
    torch = _t()
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((B * S, hidden), generator=g).to(dtype)
    w = (torch.randn((3 * H * D, hidden), generator=g) * hidden ** -0.5).to(dtype)
    return x, w


def _reference(x, w, B, S, H, D, eps, q_gain, k_gain, split, cos, sin, offset, norm, rope):
    """fp32 [3, B, H, S, D] from the oracle ops; gains are [2, D] (set 1 from
    global token split) or None."""
    y = (x.double().numpy() @ w.double().numpy().T).astype(np.float32)  # [B*S, 3HD]
    out = np.zeros((3, B, H, S, D), np.float32)
    rows = offset + np.arange(S)
    for t in range(3):
        for b in range(B):
            a = np.ascontiguousarray(y[b * S:(b + 1) * S, t * H * D:(t + 1) * H * D])
            if t < 2 and norm:
                gain = q_gain if t == 0 else k_gain
                for gs, sel in ((0, rows < split if split > 0 else rows >= 0),
                                (1, rows >= split if split > 0 else rows < 0)):
                    if sel.any():
                        part = np.ascontiguousarray(a[sel])
                        O.batch_head_norm(part, gain[gs], H, D, part.shape[0], eps)
                        a[sel] = part
            hsd = np.ascontiguousarray(a.reshape(S, H, D).transpose(1, 0, 2))
            if t < 2 and rope:
                O.mrope(hsd, cos[offset:offset + S], sin[offset:offset + S], S, H, head_dim=D)
            out[t, b] = hsd
    return out


@pytest.mark.parametrize("B,S,hidden,H,D,dtype,norm,rope,split,offset", [
    (2, 300, 256, 4, 128, "f16", True, True, 100, 7),      # 256-column tiles, ragged M
    (1, 257, 192, 4, 128, "bf16", True, True, 0, 0),       # bf16 operands
    (1, 130, 128, 3, 128, "f16", True, False, 64, 0),      # 128-column tiles (1 head)
    (2, 96, 320, 6, 64, "f16", True, False, 50, 3),        # D=64, 2 heads per tile
    (1, 64, 64, 2, 128, "f16", False, False, 0, 0),        # plain GEMM, one k block
])
def test_qkv_project_vs_oracle(ctx, B, S, hidden, H, D, dtype, norm, rope, split, offset):
    import llmr_attn as L
    torch = _t()
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    x, w = _inputs(B * 1000 + S, B, S, hidden, H, D, tdt)
    rng = np.random.default_rng(S)
    q_gain = rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)
    k_gain = rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)
    pos = np.stack([np.zeros(offset + S), np.arange(offset + S) % 17,
                    np.arange(offset + S) // 17], 1).astype(np.int32)
    axes = (16, 56, 56) if D == 128 else (16, 24, 24)
    cos, sin = L.rope_tables(pos, axes, 10000.0)
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, norm_q=norm, norm_k=norm,
                       rope=rope, split_row=split, rope_row_offset=offset, eps=1e-6)
    out = torch.empty((3, B, H, S, D), device="cuda", dtype=torch.float16)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    L.qkv_project(ctx, x.cuda(), w.cuda(), out, cfg, batch=B, seq_len=S,
                  q_gain=dev(q_gain if split > 0 else q_gain[0]) if norm else None,
                  k_gain=dev(k_gain if split > 0 else k_gain[0]) if norm else None,
                  cos=dev(cos) if rope else None, sin=dev(sin) if rope else None)
    ctx.sync()
    got = out.float().cpu().numpy()
    qg = q_gain if split > 0 else q_gain[:1].repeat(2, 0)
    kg = k_gain if split > 0 else k_gain[:1].repeat(2, 0)
    want = _reference(x, w, B, S, H, D, 1e-6, qg, kg, split, cos, sin, offset, norm, rope)
    # fp16 output: within one fp16 rounding of the fp32 result (plus the
    # different fp32 accumulation order of the GEMM)
    err = np.abs(got - want)
    bound = 1e-3 * np.abs(want) + 2e-5
    assert np.all(err <= bound), (err.max(), np.unravel_index(np.argmax(err - bound), err.shape))


def test_qkv_project_then_attention_matches_block(ctx):
    """GEMM epilogue output fed straight to the attention kernel (BHSD fp16,
    no prologue) equals the oracle's whole block on the GEMM result."""
    import llmr_attn as L
    torch = _t()
    B, S, hidden, H, D = 1, 384, 256, 4, 128
    x, w = _inputs(11, B, S, hidden, H, D, torch.float16)
    rng = np.random.default_rng(5)
    q_gain = rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)
    k_gain = rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)
    pos = np.stack([np.zeros(S), np.arange(S) // 16, np.arange(S) % 16], 1).astype(np.int32)
    cos, sin = L.rope_tables(pos, (16, 56, 56), 10000.0)
    split = 64
    cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, norm_q=True, norm_k=True,
                       rope=True, split_row=split, eps=1e-6)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    qkv = torch.empty((3, B, H, S, D), device="cuda", dtype=torch.float16)
    L.qkv_project(ctx, x.cuda(), w.cuda(), qkv, cfg, batch=B, seq_len=S, q_gain=dev(q_gain),
                  k_gain=dev(k_gain), cos=dev(cos), sin=dev(sin))
    o = torch.empty((B, S, H * D), device="cuda")
    plain = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, layout=L.BHSD)
    L.attention_fused(ctx, qkv[0], qkv[1], qkv[2], o, plain, batch=B, seq_len=S)
    ctx.sync()
    y = (x.double().numpy() @ w.double().numpy().T).astype(np.float32)
    hd = H * D
    want = O.attention_block(y[:, :hd], y[:, hd:2 * hd], y[:, 2 * hd:], H, D, D ** -0.5,
                             eps=1e-6, q_gain=q_gain, k_gain=k_gain, split_row=split,
                             cos=cos, sin=sin)
    err = np.abs(o[0].cpu().numpy().astype(np.float64) - want)
    assert err.max() <= 2e-3 and err.mean() <= 2e-4, (err.max(), err.mean())


def test_qkv_project_rejects_bad_shapes(ctx):
    import llmr_attn as L
    torch = _t()
    x = torch.zeros((64, 96), device="cuda", dtype=torch.float16)      # hidden % 64 != 0
    w = torch.zeros((3 * 128, 96), device="cuda", dtype=torch.float16)
    out = torch.empty((3, 1, 1, 64, 128), device="cuda", dtype=torch.float16)
    cfg = L.AttnConfig(n_heads=1, head_dim=128, scale=0.1)
    with pytest.raises(L.LlmrError) as ei:
        L.qkv_project(ctx, x, w, out, cfg, batch=1, seq_len=64)
    assert ei.value.status == L.EINVAL
    xb = torch.zeros((64, 128), device="cuda", dtype=torch.bfloat16)
    w16 = torch.zeros((3 * 128, 128), device="cuda", dtype=torch.float16)
    with pytest.raises(L.LlmrError):
        L.qkv_project(ctx, xb, w16, out, cfg, batch=1, seq_len=64)   # mixed dtypes


# ------------------------------------------------------------------ out projection

@pytest.mark.parametrize("B,S,in_dim,out_dim,split,dtype,with_bias,with_gate", [
    (1, 300, 256, 512, 100, "f16", True, True),     # two streams, ragged segments
    (2, 257, 192, 256, 0, "bf16", False, True),     # one stream, bf16, batch 2
    (1, 128, 64, 768, 64, "bf16", True, False),     # one k block, three column tiles
])
def test_out_project_vs_numpy(ctx, B, S, in_dim, out_dim, split, dtype, with_bias, with_gate):
    """hidden += gate_g * (o . w_g^T + bias_g), g by token index: the
    reference's matmul + broadcast_bias_add + gated_residual_add per stream."""
    import llmr_attn as L
    torch = _t()
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    g = torch.Generator().manual_seed(S + out_dim)
    o = torch.randn((B * S, in_dim), generator=g).to(tdt)
    w = [(torch.randn((out_dim, in_dim), generator=g) * in_dim ** -0.5).to(tdt) for _ in range(2)]
    bias = [torch.randn(out_dim, generator=g) if with_bias else None for _ in range(2)]
    gate = [torch.rand(out_dim, generator=g) + 0.5 if with_gate else None for _ in range(2)]
    hidden = torch.randn((B * S, out_dim), generator=g)
    want = hidden.double().clone()
    for b in range(B):
        for s0, s1, k in ((0, split if split else S, 0), (split, S, 1)) if split else ((0, S, 0),):
            rows = slice(b * S + s0, b * S + s1)
            y = o[rows].double() @ w[k].double().t()
            if bias[k] is not None:
                y = y + bias[k].double()
            if gate[k] is not None:
                y = y * gate[k].double()
            want[rows] += y
    cu = lambda t: None if t is None else t.cuda()
    hd = hidden.cuda()
    L.out_project(ctx, o.cuda(), hd, cu(w[0]), cu(w[1]) if split else None, batch=B, seq_len=S,
                  split_row=split, bias0=cu(bias[0]), bias1=cu(bias[1]), gate0=cu(gate[0]),
                  gate1=cu(gate[1]))
    ctx.sync()
    err = (hd.cpu().double() - want).abs()
    assert err.max().item() < 2e-4 * max(1.0, want.abs().max().item()), err.max().item()


def test_out_project_rejects_bad_shapes(ctx):
    import llmr_attn as L
    torch = _t()
    o = torch.zeros((64, 128), device="cuda", dtype=torch.float16)
    w = torch.zeros((200, 128), device="cuda", dtype=torch.float16)     # out_dim % 256
    h = torch.zeros((64, 200), device="cuda")
    with pytest.raises(L.LlmrError) as ei:
        L.out_project(ctx, o, h, w, batch=1, seq_len=64)
    assert ei.value.status == L.EINVAL
    w2 = torch.zeros((256, 128), device="cuda", dtype=torch.float16)
    h2 = torch.zeros((64, 256), device="cuda")
    with pytest.raises(L.LlmrError):        # a split without the second weight set
        L.out_project(ctx, o, h2, w2, batch=1, seq_len=64, split_row=32)
