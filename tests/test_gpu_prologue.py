"""GPU: the streaming prologue (the default for 16-byte aligned inputs) writes
exactly what the one-(tensor, head)-per-CTA prologue writes, bit for bit, for
Q/K/V of every input dtype, D = 64 and 128, ragged token counts, the txt/img
gain split, a RoPE row offset, BSHD and strided BHSD inputs. The two kernels
are selected per process (LLMR_PROLOGUE_LEGACY), so each runs in a child
process on the same seeded inputs."""
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
D, S, H, B, ind, layout, out = int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), \
    int(sys.argv[5]), sys.argv[6], sys.argv[7], sys.argv[8]
tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[ind]
rng = np.random.default_rng(D * 1000 + S)
bhsd = layout == "bhsd"
pad = 8 if bhsd else 0
shape = (B, H, S, D + pad) if bhsd else (B, S, H, D)
mk = lambda: torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).cuda().to(tdt)
q, k, v = mk(), mk(), mk()
qg = torch.from_numpy(rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)).cuda()
kg = torch.from_numpy(rng.uniform(0.8, 1.2, (2, D)).astype(np.float32)).cuda()
off = 37
ids = C.flux_ids(100, 72, 72)[: S + off]
assert ids.shape[0] == S + off
axes = (16, 56, 56) if D == 128 else (16, 24, 24)
cos, sin = (torch.from_numpy(t).cuda() for t in L.rope_tables(ids, axes, 1e4))
cfg = L.AttnConfig(n_heads=H, head_dim=D, scale=D ** -0.5, eps=1e-6, norm_q=True, norm_k=True,
                   rope=True, split_row=100, rope_row_offset=off,
                   layout=L.BHSD if bhsd else L.BSHD)
strides = None
if bhsd:
    rs = D + pad
    strides = {f"{t}_{n}": v for t in "qkv" for n, v in
               (("row_stride", rs), ("head_stride", S * rs), ("batch_stride", H * S * rs))}
res = torch.empty((3, B, H, S, D), device="cuda", dtype=torch.float16)
ctx = L.Context(0)
L.attention_prologue(ctx, q, k, v, res, cfg, batch=B, seq_len=S, q_gain=qg, k_gain=kg,
                     cos=cos, sin=sin, strides=strides)
ctx.sync()
np.save(out, res.cpu().view(torch.int16).numpy())
"""

CASES = [(128, 4608, 3, 1, "bf16", "bshd"), (128, 1000, 5, 2, "f32", "bshd"),
         (64, 1370, 4, 1, "f16", "bshd"), (64, 77, 3, 3, "bf16", "bhsd"),
         (128, 333, 30, 1, "bf16", "bhsd"), (64, 5, 1, 1, "f32", "bshd")]


@pytest.mark.parametrize("D,S,H,B,ind,layout", CASES)
def test_stream_prologue_bit_exact_with_legacy(tmp_path, D, S, H, B, ind, layout):
    outs = []
    for legacy in (False, True):
        env = dict(os.environ)
        env.pop("LLMR_PROLOGUE_LEGACY", None)
        if legacy:
            env["LLMR_PROLOGUE_LEGACY"] = "1"
        out = str(tmp_path / f"p{int(legacy)}.npy")
        subprocess.run([sys.executable, "-c", CHILD, ROOT, str(D), str(S), str(H), str(B), ind,
                        layout, out], check=True, env=env, timeout=300)
        outs.append(np.load(out))
    assert np.array_equal(outs[0], outs[1])
