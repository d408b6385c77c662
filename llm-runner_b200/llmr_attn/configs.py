"""The five benchmark/parity configurations of the attention path and their
seeded synthetic inputs.

Position ids follow the reference's host table builders
(dependencies/flux.c3l/flux_dit.c3:396-525 for Flux: text tokens first,
image tokens at (t, h, w) on their patch grid; dependencies/zimage.c3l/
dit.c3:561-757 for Z-Image: text tokens 1-indexed on axis 0) with each
configuration's own axes, theta and grids. Where a configuration leaves an id
unstated, the choice made here is recorded in the `ids_note` field.

Seeded inputs: numpy PCG64 `default_rng(seed)`, `standard_normal(float32)`
drawn in the order Q, K, V (each [B, S, H, D]), then q_gain, k_gain; then
rounded to the configuration dtype (RNE). The oracle and the GPU path consume
exactly those rounded values.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Tuple

import numpy as np


@dataclass(frozen=True)
class AttnCase:
    name: str
    batch: int
    n_heads: int
    seq_len: int
    head_dim: int
    dtype: str                   # "f32" | "f16" | "bf16"
    seed: int
    scale: float
    input_scale: float = 1.0     # Q/K/V ~ N(0,1) * input_scale
    norm: bool = False
    eps: float = 1e-6
    gain: str = "none"           # "none" | "one" | "uniform"
    split_row: int = 0           # txt/img gain split (0 = one gain set)
    rope: Optional[Tuple] = None  # (axes_dims, theta)
    exact: bool = False          # spatial_attention math (fp32, exact softmax)
    layout: str = "bshd"
    ids_note: str = ""
    tol_max: float = 2e-3
    tol_mean: float = 2e-4

    @property
    def flops(self) -> float:
        return 4.0 * self.batch * self.n_heads * self.seq_len ** 2 * self.head_dim

    @property
    def elem_bytes(self) -> int:
        return 4 if self.dtype == "f32" else 2

    @property
    def io_bytes(self) -> int:
        """Algorithmic HBM bytes: Q, K, V read once and O written once."""
        return 4 * self.batch * self.n_heads * self.seq_len * self.head_dim * self.elem_bytes


def flux_ids(n_txt: int, gh: int, gw: int) -> np.ndarray:
    """Text (0,0,0); image (0,h,w) row-major over the patch grid."""
    ids = np.zeros((n_txt + gh * gw, 3), np.int32)
    hh, ww = np.meshgrid(np.arange(gh), np.arange(gw), indexing="ij")
    ids[n_txt:, 1] = hh.reshape(-1)
    ids[n_txt:, 2] = ww.reshape(-1)
    return ids


def zimage_ids(n_txt: int, gh: int, gw: int) -> np.ndarray:
    """Text (t+1,0,0) as the reference's 1-indexed text axis (dit.c3:675-682);
    image (0,h,w) as the configuration states."""
    ids = flux_ids(n_txt, gh, gw)
    ids[:n_txt, 0] = np.arange(1, n_txt + 1)
    return ids


def qwen_ids(n_txt: int, gh: int, gw: int, n_frames: int) -> np.ndarray:
    """Text (0,0,0); frame f image tokens (f,h,w) on their own grid."""
    parts = [np.zeros((n_txt, 3), np.int32)]
    hh, ww = np.meshgrid(np.arange(gh), np.arange(gw), indexing="ij")
    for f in range(n_frames):
        blk = np.zeros((gh * gw, 3), np.int32)
        blk[:, 0] = f
        blk[:, 1] = hh.reshape(-1)
        blk[:, 2] = ww.reshape(-1)
        parts.append(blk)
    return np.concatenate(parts)


C1 = AttnCase("plumbing", 1, 4, 256, 64, "f32", seed=0, scale=1 / 8, exact=True,
              layout="bhsd", tol_max=1e-5, tol_mean=1e-5)
C2 = AttnCase("depth_vitl", 1, 16, 1370, 64, "f16", seed=1, scale=1 / 8, input_scale=0.5,
              exact=False)
C3 = AttnCase("flux_1024", 1, 24, 4608, 128, "bf16", seed=2, scale=128 ** -0.5, norm=True,
              eps=1e-6, gain="uniform", split_row=512, rope=((16, 56, 56), 10000.0),
              ids_note="text (0,0,0), image (0,h,w) on 64x64")
C4 = AttnCase("zimage_cfg", 2, 30, 4352, 128, "bf16", seed=3, scale=128 ** -0.5, norm=True,
              eps=1e-5, gain="one", rope=((32, 48, 48), 256.0),
              ids_note="text (t+1,0,0) [reference convention], image (0,h,w) on 64x64")
C5 = AttnCase("qwen_edit_2048", 1, 24, 33792, 128, "bf16", seed=4, scale=128 ** -0.5,
              norm=True, eps=1e-6, gain="uniform", split_row=1024,
              rope=((16, 56, 56), 10000.0),
              ids_note="text (0,0,0), target (0,h,w), reference (1,h,w) on 128x128")
CASES = {c.name: c for c in (C1, C2, C3, C4, C5)}


def case_ids(case: AttnCase) -> Optional[np.ndarray]:
    if case.rope is None:
        return None
    if case.name == "flux_1024":
        return flux_ids(512, 64, 64)
    if case.name == "zimage_cfg":
        return zimage_ids(256, 64, 64)
    if case.name == "qwen_edit_2048":
        return qwen_ids(1024, 128, 128, 2)
    raise KeyError(case.name)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 values to the config dtype (RNE) and widen back to fp32."""
    if dtype == "f32":
        return x.astype(np.float32)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def make_inputs(case: AttnCase, seq_len: Optional[int] = None, batch: Optional[int] = None,
                n_heads: Optional[int] = None):
    """Seeded inputs in BSHD [B,S,H,D] fp32 (already rounded to case.dtype) and
    gains. Overrides shrink a case for fast tests with the same recipe."""
    S = seq_len or case.seq_len
    B = batch or case.batch
    H = n_heads or case.n_heads
    rng = np.random.default_rng(case.seed)
    shape = (B, S, H, case.head_dim)
    q = rng.standard_normal(shape, dtype=np.float32) * np.float32(case.input_scale)
    k = rng.standard_normal(shape, dtype=np.float32) * np.float32(case.input_scale)
    v = rng.standard_normal(shape, dtype=np.float32) * np.float32(case.input_scale)
    q, k, v = (round_to(t, case.dtype) for t in (q, k, v))
    nsets = 2 if case.split_row else 1
    if case.gain == "uniform":
        qg = rng.uniform(0.8, 1.2, size=(nsets, case.head_dim)).astype(np.float32)
        kg = rng.uniform(0.8, 1.2, size=(nsets, case.head_dim)).astype(np.float32)
    elif case.gain == "one":
        qg = np.ones((nsets, case.head_dim), np.float32)
        kg = np.ones((nsets, case.head_dim), np.float32)
    else:
        qg = kg = None
    return q, k, v, qg, kg


def split_for(case: AttnCase, seq_len: int) -> int:
    """txt/img split row for a (possibly shortened) case."""
    return min(case.split_row, seq_len)


@dataclass
class Prepared:
    """Host-side arrays for one case (BSHD fp32 values + tables)."""
    case: AttnCase
    q: np.ndarray
    k: np.ndarray
    v: np.ndarray
    q_gain: Optional[np.ndarray]
    k_gain: Optional[np.ndarray]
    cos: Optional[np.ndarray] = None
    sin: Optional[np.ndarray] = None
    extra: dict = field(default_factory=dict)


def prepare(case: AttnCase, rope_tables_fn, seq_len: Optional[int] = None,
            batch: Optional[int] = None, n_heads: Optional[int] = None) -> Prepared:
    q, k, v, qg, kg = make_inputs(case, seq_len, batch, n_heads)
    cos = sin = None
    if case.rope is not None:
        ids = case_ids(case)[: q.shape[1]]
        cos, sin = rope_tables_fn(ids, case.rope[0], case.rope[1])
    return Prepared(case, q, k, v, qg, kg, cos, sin)
