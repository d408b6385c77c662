"""GPU: the prologue fused into the attention kernel (LLMR_FUSED_PROLOGUE=1;
measured slower than the two-kernel default, kept as an option) gives exactly the output of the two-kernel path (prologue kernel,
then the attention kernel), bit for bit: O in every output dtype and the
LSE, for bf16 / fp16 inputs, D = 64 and 128, batch 2, ragged token counts,
the txt/img gain split, a RoPE row offset, strided BHSD inputs, a long
sequence where the start-up phase covers few heads, and a grid where each
CTA runs up to seven units (the background writer runs far ahead). The two paths are
selected per process (LLMR_FUSED_PROLOGUE), so each runs in a child
process on the same seeded inputs; the fused path is also checked to be one
launch."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1] + "/llm-runner_b200")
import llmr_attn as L
from llmr_attn import configs as C
D, S, H, B = (int(x) for x in sys.argv[2:6])
ind, outd, layout, norm, out = sys.argv[6], sys.argv[7], sys.argv[8], sys.argv[9] == "1", sys.argv[10]
tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
g = torch.Generator(device="cuda").manual_seed(D * 7919 + S * 31 + H)
bhsd = layout == "bhsd"
pad = 8 if bhsd else 0
shape = (B, H, S, D + pad) if bhsd else (B, S, H, D)
q, k, v = (torch.randn(shape, device="cuda", generator=g).to(tdt[ind]) for _ in range(3))
qg = (0.8 + 0.4 * torch.rand((2, D), device="cuda", generator=g)).float()
kg = (0.8 + 0.4 * torch.rand((2, D), device="cuda", generator=g)).float()
off = 21
ids = C.qwen_ids(100, 200, 200, 1)[: S + off]
assert ids.shape[0] == S + off
axes = (16, 56, 56) if D == 128 else (16, 24, 24)
cos, sin = (torch.from_numpy(t).cuda() for t in L.rope_tables(ids, axes, 1e4))
cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, eps=1e-6, norm_q=norm, norm_k=norm,
                   rope=True, split_row=100, rope_row_offset=off,
                   layout=L.BHSD if bhsd else L.BSHD)
strides = None
if bhsd:
    rs = D + pad
    strides = {f"{t}_{n}": v for t in "qkv" for n, v in
               (("row_stride", rs), ("head_stride", S * rs), ("batch_stride", H * S * rs))}
o = torch.full((B, S, H * D), float("nan"), device="cuda", dtype=tdt[outd])
lse = torch.full((B, H, S), float("nan"), device="cuda")
ctx = L.Context(0)
ctx.reserve(L.workspace_bytes(L.make_desc(cfg, B, S, L._dtype_code(q), L._dtype_code(o))))
for _ in range(2):  # twice: the piece counters must be clean for the second launch
    n0 = ctx.launches
    L.attention_fused(ctx, q, k, v, o, cfg, batch=B, seq_len=S, q_gain=qg if norm else None,
                      k_gain=kg if norm else None, cos=cos, sin=sin, lse=lse, strides=strides)
    ctx.sync()
    launches = ctx.launches - n0
assert torch.isfinite(o.float()).all() and torch.isfinite(lse).all()
np.savez(out, o=o.float().cpu().numpy(), lse=lse.cpu().numpy(), launches=launches)
"""

CASES = [
    (128, 4608, 24, 1, "bf16", "bf16", "bshd", 1),   # the Flux shape
    (128, 1000, 5, 2, "f16", "f32", "bshd", 1),
    (64, 1370, 4, 1, "bf16", "f16", "bshd", 1),
    (64, 77, 3, 3, "f16", "f32", "bhsd", 1),
    (128, 333, 30, 1, "bf16", "f32", "bhsd", 1),
    (128, 700, 2, 1, "bf16", "f32", "bshd", 0),     # RoPE without norm
    (128, 33792, 2, 1, "bf16", "f32", "bshd", 1),   # long: start-up covers one head
    (64, 8192, 16, 2, "f16", "bf16", "bshd", 1),    # 1024 units: up to 7 per CTA
]


@pytest.mark.parametrize("D,S,H,B,ind,outd,layout,norm", CASES)
def test_fused_prologue_bit_exact_with_two_kernels(tmp_path, D, S, H, B, ind, outd, layout, norm):
    res = []
    for separate in (False, True):
        env = dict(os.environ)
        env.pop("LLMR_FUSED_PROLOGUE", None)
        if not separate:
            env["LLMR_FUSED_PROLOGUE"] = "1"
        out = str(tmp_path / f"r{int(separate)}.npz")
        subprocess.run([sys.executable, "-c", CHILD, ROOT, str(D), str(S), str(H), str(B), ind,
                        outd, layout, str(norm), out], check=True, env=env, timeout=600)
        res.append(np.load(out))
    fused, two = res
    assert int(fused["launches"]) == 1 and int(two["launches"]) == 2
    assert np.array_equal(fused["o"], two["o"])
    assert np.array_equal(fused["lse"], two["lse"])
