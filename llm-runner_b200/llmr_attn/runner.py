"""Device-side driver for one attention case: uploads a `configs.Prepared`
case and runs the fused op on it. Used by the benchmark and the tests; the op
itself is `llmr_attn.attention_fused`."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

import llmr_attn as L
from llmr_attn.configs import AttnCase, Prepared

_TORCH = None


def _torch():
    global _TORCH
    if _TORCH is None:
        import torch
        _TORCH = torch
    return _TORCH


def torch_dtype(name: str):
    t = _torch()
    return {"f32": t.float32, "f16": t.float16, "bf16": t.bfloat16}[name]


def attn_config(case: AttnCase, seq_len: int) -> L.AttnConfig:
    return L.AttnConfig(
        n_heads=case.n_heads, head_dim=case.head_dim, scale=case.scale,
        layout=L.BHSD if case.layout == "bhsd" else L.BSHD, eps=case.eps,
        norm_q=case.norm, norm_k=case.norm, rope=case.rope is not None,
        exact=case.exact, split_row=min(case.split_row, seq_len))


@dataclass
class DeviceCase:
    """Device-resident inputs/outputs of one case, ready to run repeatedly."""
    cfg: L.AttnConfig
    batch: int
    seq_len: int
    q: object
    k: object
    v: object
    o: object
    q_gain: Optional[object]
    k_gain: Optional[object]
    cos: Optional[object]
    sin: Optional[object]
    lse: Optional[object] = None

    def run(self, ctx: L.Context) -> None:
        L.attention_fused(ctx, self.q, self.k, self.v, self.o, self.cfg, batch=self.batch,
                          seq_len=self.seq_len, q_gain=self.q_gain, k_gain=self.k_gain,
                          cos=self.cos, sin=self.sin, lse=self.lse)

    def desc(self) -> L.AttnDesc:
        return L.make_desc(self.cfg, self.batch, self.seq_len, L._dtype_code(self.q),
                           L._dtype_code(self.o), lse=self.lse is not None)


def to_device(prep: Prepared, device: int = 0, out_dtype: Optional[str] = None,
              with_lse: bool = False, n_heads: Optional[int] = None) -> DeviceCase:
    """Uploads a prepared case. Inputs keep their BSHD [B,S,H,D] layout (or
    BHSD for a case whose layout says so); O is [B,S,H*D]."""
    t = _torch()
    case = prep.case
    dt = torch_dtype(case.dtype)
    dev = f"cuda:{device}"
    B, S, H, D = prep.q.shape
    def up(a):
        x = t.from_numpy(np.ascontiguousarray(a))
        if case.layout == "bhsd":
            x = x.permute(0, 2, 1, 3).contiguous()
        return x.to(dev).to(dt)
    q, k, v = up(prep.q), up(prep.k), up(prep.v)
    od = torch_dtype(out_dtype or ("f32" if case.exact else case.dtype))
    o = t.empty((B, S, H * D), dtype=od, device=dev)
    g = lambda a: None if a is None else t.from_numpy(np.ascontiguousarray(a)).to(dev)
    cfg = attn_config(case, S)
    cfg.n_heads = H
    lse = t.empty((B, H, S), dtype=t.float32, device=dev) if with_lse else None
    return DeviceCase(cfg, B, S, q, k, v, o, g(prep.q_gain), g(prep.k_gain), g(prep.cos),
                      g(prep.sin), lse)
