"""ctypes binding of the CPU oracle (oracle/liboracle_attn.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs, never by the shipped package.
PARITY UNPINNED: the reference has no golden vectors for this path and cannot
be built here; see attn_oracle.h.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle_attn.so")


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load():
    if not os.path.exists(LIB):
        build()
    lib = ctypes.CDLL(LIB)
    vp, u32, f32, i32, f64 = (ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float,
                              ctypes.c_int, ctypes.c_double)
    sig = {
        "orc_round_f16": (f32, [f32]),
        "orc_set_threads": (None, [ctypes.c_int]),
        "orc_round_bf16": (f32, [f32]),
        "orc_batch_head_norm": (None, [vp, vp, u32, u32, u32, f32]),
        "orc_transpose_heads": (None, [vp, vp, u32, u32, u32, u32]),
        "orc_mrope": (None, [vp, vp, vp, u32, u32, u32]),
        "orc_flash_attention_v2": (None, [vp, vp, vp, vp, u32, u32, u32, f32, u32, u32, i32]),
        "orc_spatial_attention": (None, [vp, vp, vp, vp, u32, u32, u32, f32, u32, u32, i32]),
        "orc_vae_attention": (None, [vp, vp, vp, vp, u32, u32, u32, f32, u32, u32, u32, i32]),
        "orc_split_qkv": (None, [vp, vp, vp, vp, u32, u32]),
        "orc_rope_tables": (None, [vp, u32, u32, vp, f32, vp, vp]),
        "orc_attention_block": (None, [vp, vp, vp, vp, u32, u32, u32, f32, f32, vp, vp, vp,
                                       vp, u32, vp, vp, i32, u32, u32, i32]),
        "orc_attention_f64": (None, [vp, vp, vp, vp, u32, u32, u32, f64, u32, u32, i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a):
    return None if a is None else a.ctypes.data


def set_threads(n: int) -> None:
    """OpenMP threads for all later oracle calls (0 keeps the default)."""
    lib.orc_set_threads(int(n))


def round_f16(x: float) -> float:
    return lib.orc_round_f16(x)


def round_bf16(x: float) -> float:
    return lib.orc_round_bf16(x)


def batch_head_norm(data, gain, n_heads, head_dim, seq_len, eps):
    """In place on a float32 C-contiguous array [S, H*D]."""
    assert data.dtype == np.float32 and data.flags.c_contiguous
    g = _c(gain)
    lib.orc_batch_head_norm(data.ctypes.data, g.ctypes.data, n_heads, head_dim, seq_len, eps)


def transpose_heads(inp, seq_len, n_heads, head_dim, direction):
    inp = _c(inp)
    out = np.empty_like(inp)
    lib.orc_transpose_heads(inp.ctypes.data, out.ctypes.data, seq_len, n_heads, head_dim,
                            direction)
    return out


def mrope(data, cos, sin, seq_len, n_heads, head_dim=128):
    assert data.dtype == np.float32 and data.flags.c_contiguous
    c, s = _c(cos), _c(sin)
    lib.orc_mrope(data.ctypes.data, c.ctypes.data, s.ctypes.data, seq_len, n_heads, head_dim)


def flash_attention_v2(q, k, v, head_dim, n_heads, seq_len, scale, qb_range=None,
                       threads=0):
    """q,k,v [H,S,D] -> O [S, H*D] (rows outside qb_range are zero)."""
    q, k, v = _c(q), _c(k), _c(v)
    o = np.zeros((seq_len, n_heads * head_dim), np.float32)
    b0, b1 = qb_range or (0, 0xFFFFFFFF)
    lib.orc_flash_attention_v2(q.ctypes.data, k.ctypes.data, v.ctypes.data, o.ctypes.data,
                               head_dim, n_heads, seq_len, scale, b0, b1, threads)
    return o


def spatial_attention(q, k, v, head_dim, n_heads, seq_len, scale, rows=None, threads=0):
    """q,k,v [H,S,D] -> O [H,S,D] (rows outside `rows` are zero)."""
    q, k, v = _c(q), _c(k), _c(v)
    o = np.zeros((n_heads, seq_len, head_dim), np.float32)
    r0, r1 = rows or (0, seq_len)
    lib.orc_spatial_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, o.ctypes.data,
                              head_dim, n_heads, seq_len, scale, r0, r1, threads)
    return o


def vae_attention(q, k, v, head_dim, n_heads, seq_len, scale, channels=None, rows=None,
                  threads=0):
    """q,k,v [S, C] -> O [S, C] (rows outside `rows` are zero); C defaults to
    n_heads * head_dim."""
    q, k, v = _c(q), _c(k), _c(v)
    channels = channels or n_heads * head_dim
    o = np.zeros((seq_len, channels), np.float32)
    r0, r1 = rows or (0, seq_len)
    lib.orc_vae_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, o.ctypes.data,
                          head_dim, n_heads, seq_len, scale, channels, r0, r1, threads)
    return o


def split_qkv(qkv, dim, n_rows):
    qkv = _c(qkv)
    q = np.empty((n_rows, dim), np.float32)
    k = np.empty_like(q)
    v = np.empty_like(q)
    lib.orc_split_qkv(qkv.ctypes.data, q.ctypes.data, k.ctypes.data, v.ctypes.data, dim,
                      n_rows)
    return q, k, v


def rope_tables(pos, axes_dims, theta):
    pos = _c(pos, np.int32)
    axes = _c(axes_dims, np.uint32)
    S = pos.shape[0]
    half = int(axes.sum()) // 2
    cos = np.empty((S, half), np.float32)
    sin = np.empty((S, half), np.float32)
    lib.orc_rope_tables(pos.ctypes.data, S, len(axes), axes.ctypes.data, theta,
                        cos.ctypes.data, sin.ctypes.data)
    return cos, sin


def attention_block(q, k, v, n_heads, head_dim, scale, eps=1e-6, q_gain=None, k_gain=None,
                    split_row=0, cos=None, sin=None, exact=False, rows=None, threads=0):
    """One batch element of the reference's block sequence.

    q,k,v: [S, H*D] (BSHD of one batch element). q_gain/k_gain: [D] or [2,D]
    (gain set 0 for rows < split_row, set 1 after). Returns O [S, H*D]; only
    rows in `rows` (rounded out to 16-row blocks for flash_attention_v2) are
    computed, the rest are zero.
    """
    S = q.shape[0]
    q, k, v = _c(q).reshape(S, -1), _c(k).reshape(S, -1), _c(v).reshape(S, -1)
    o = np.zeros((S, n_heads * head_dim), np.float32)

    def gains(g):
        if g is None:
            return None, None
        g = _c(g).reshape(-1, head_dim)
        return g[0].copy(), (g[1].copy() if g.shape[0] > 1 else None)

    qg0, qg1 = gains(q_gain)
    kg0, kg1 = gains(k_gain)
    c = None if cos is None else _c(cos)
    s = None if sin is None else _c(sin)
    r0, r1 = rows or (0, S)
    lib.orc_attention_block(q.ctypes.data, k.ctypes.data, v.ctypes.data, o.ctypes.data, S,
                            n_heads, head_dim, scale, eps, _p(qg0), _p(qg1), _p(kg0),
                            _p(kg1), split_row if qg1 is not None else 0, _p(c), _p(s),
                            1 if exact else 0, r0, r1, threads)
    return o


def attention_f64(q, k, v, head_dim, n_heads, seq_len, scale, rows=None, threads=0):
    """fp64 exact attention on [H,S,D] fp32 inputs -> [H,S,D] float64."""
    q, k, v = _c(q), _c(k), _c(v)
    o = np.zeros((n_heads, seq_len, head_dim), np.float64)
    r0, r1 = rows or (0, seq_len)
    lib.orc_attention_f64(q.ctypes.data, k.ctypes.data, v.ctypes.data, o.ctypes.data,
                          head_dim, n_heads, seq_len, scale, r0, r1, threads)
    return o
