"""Generates the golden vectors in tests/golden/ from an independent numpy
restatement of the reference shaders.

The reference ships no golden vectors for this path and cannot be run here
(C3 + Slang + Vulkan), so these fixtures are produced by a second restatement
written separately from oracle/attn_oracle.cpp, from the same shader sources:
  dependencies/zimage.c3l/shaders/flash_attn.slang:38-241   (flash_attention_v2)
  dependencies/zimage.c3l/shaders/zimage.slang:575-601, :623-659
  dependencies/zimage.c3l/shaders/mrope.slang:33-54
  lib/shaders/diffusion.slang:478-569                        (spatial_attention)
  lib/shaders/diffusion.slang:1846-1975                      (vae_attention)
  test/mesh_encoder_test.c3:95-135       (cpu_attention, the reference's own
                                          CPU check of its FA2-style kernel)
  test/mesh_encoder_test.c3:81-92        (cpu_rmsnorm)
  dependencies/depth_anything.c3l/shaders/depth.slang:40-58  (split_qkv)
  dependencies/flux.c3l/flux_dit.c3:461-497                  (RoPE tables)
Two restatements agreeing is what the oracle is checked against.

Files use the reference's dump format (test/README.md:64-68): the 16-byte
header b"C3_DEBUG_TENSOR\\0" followed by raw little-endian float32. Shapes and
parameters are in manifest.json. Run: python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
HEADER = b"C3_DEBUG_TENSOR\x00"
f32 = np.float32


def save(name, arr):
    arr = np.ascontiguousarray(arr, dtype=np.float32)
    with open(os.path.join(HERE, name + ".bin"), "wb") as fh:
        fh.write(HEADER)
        fh.write(arr.tobytes())
    return {"file": name + ".bin", "shape": list(arr.shape)}


def to_f16(x):
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------- restatements
def np_head_norm(data, gain, H, D, S, eps):
    """zimage.slang:623-659 (per-thread squares, 256-wide tree sum)."""
    out = data.reshape(S, H, D).copy()
    for pos in range(S):
        for h in range(H):
            x = out[pos, h]
            sh = np.zeros(256, f32)
            sh[:D] = x * x
            s = 128
            while s > 0:
                sh[:s] = sh[:s] + sh[s:2 * s]
                s //= 2
            rms = f32(1.0) / np.sqrt(sh[0] / f32(D) + f32(eps), dtype=f32)
            out[pos, h] = (x * rms) * gain
    return out.reshape(S, H * D)


def np_transpose(inp, S, H, D, direction):
    if direction == 0:
        return inp.reshape(S, H, D).transpose(1, 0, 2).copy()
    return inp.reshape(H, S, D).transpose(1, 0, 2).copy()


def np_mrope(data, cos, sin, S, H):
    x = data.reshape(H, S, 64, 2)
    x0, x1 = x[..., 0].copy(), x[..., 1].copy()
    out = np.empty_like(x)
    out[..., 0] = x0 * cos[None] - x1 * sin[None]
    out[..., 1] = x0 * sin[None] + x1 * cos[None]
    return out.reshape(H, S, 128)


def np_tables(pos, axes, theta):
    S = pos.shape[0]
    cols_c, cols_s = [], []
    for a, d in enumerate(axes):
        k = np.arange(d // 2, dtype=f32)
        freq = f32(1.0) / np.power(f32(theta), (f32(2) * k) / f32(d), dtype=f32)
        ang = pos[:, a:a + 1].astype(f32) * freq[None, :]
        cols_c.append(np.cos(ang, dtype=f32))
        cols_s.append(np.sin(ang, dtype=f32))
    return np.concatenate(cols_c, 1), np.concatenate(cols_s, 1)


def np_fa2(Q, K, V, D, H, S, scale):
    """flash_attn.slang:38-241 with BR=16, BC=32, fp16 operands."""
    BR, BC, DP = 16, 32, D // 2
    O = np.zeros((S, H * D), f32)
    for h in range(H):
        q16 = to_f16(Q[h])
        k16 = to_f16(K[h])
        v16 = to_f16(V[h])
        for qb in range((S + BR - 1) // BR):
            rows = np.arange(qb * BR, qb * BR + BR)
            qv = rows < S
            qt = np.zeros((BR, D), f32)
            qt[qv] = q16[rows[qv]]
            m = np.full(BR, -1.0e30, f32)
            l = np.zeros(BR, f32)
            acc = np.zeros((BR, D), f32)
            for kb in range((S + BC - 1) // BC):
                cols = np.arange(kb * BC, kb * BC + BC)
                kvv = cols < S
                kt = np.zeros((BC, D), f32)
                vt = np.zeros((BC, D), f32)
                kt[kvv] = k16[cols[kvv]]
                vt[kvv] = v16[cols[kvv]]
                dot = np.zeros((BR, BC), f32)
                for dp in range(DP):
                    t = (qt[:, None, 2 * dp] * kt[None, :, 2 * dp]
                         + qt[:, None, 2 * dp + 1] * kt[None, :, 2 * dp + 1])
                    dot = dot + t
                valid = qv[:, None] & kvv[None, :]
                s = np.where(valid, dot * f32(scale), f32(-1.0e30)).astype(f32)
                m_new = np.maximum(m, s.max(1))
                e = np.where(valid, np.exp(s - m_new[:, None], dtype=f32), f32(0))
                red = e.copy()
                w = 16
                while w > 0:
                    red[:, :w] = red[:, :w] + red[:, w:2 * w]
                    w //= 2
                r = np.exp(m - m_new, dtype=f32)
                l = r * l + red[:, 0]
                m = m_new
                new = np.zeros((BR, D), f32)
                for kv in range(BC):
                    new = new + e[:, kv:kv + 1] * vt[kv][None, :]
                acc = acc * r[:, None] + new
            for i, row in enumerate(rows):
                if row < S:
                    O[row, h * D:(h + 1) * D] = acc[i] * (f32(1.0) / l[i])
    return O


def np_spatial(Q, K, V, D, H, S, scale):
    """diffusion.slang:478-569 (exact fp32 softmax)."""
    O = np.zeros((H, S, D), f32)
    for h in range(H):
        for qp in range(S):
            dot = np.zeros(S, f32)
            for d in range(D):
                dot = dot + Q[h, qp, d] * K[h, :, d]
            sc = dot * f32(scale)
            gmax = sc.max()
            ev = np.exp(sc - gmax, dtype=f32)
            part = np.zeros(256, f32)
            for i in range(S):
                part[i % 256] = part[i % 256] + ev[i]
            w = 128
            while w > 0:
                part[:w] = part[:w] + part[w:2 * w]
                w //= 2
            p = ev / part[0]
            acc = np.zeros(D, f32)
            for pos in range(S):
                acc = acc + p[pos] * V[h, pos]
            O[h, qp] = acc
    return O


def np_cpu_attention(Q, K, V, D, H, S, scale):
    """The reference test suite's CPU attention (test/mesh_encoder_test.c3:
    95-135) on [H, S, D]: fp32 dot products summed over d in order, scores
    scaled, the row max, exp(s - max), the total summed over keys in order,
    and out = (sum_s p_s v_s, s in order) / total. All queries at once."""
    O = np.zeros((H, S, D), f32)
    for h in range(H):
        dot = np.zeros((S, S), f32)
        for d in range(D):
            dot = dot + Q[h, :, d][:, None] * K[h, :, d][None, :]
        sc = dot * f32(scale)
        top = sc.max(axis=1, keepdims=True)
        e = np.exp(sc - top, dtype=f32)
        total = np.add.accumulate(e, axis=1, dtype=f32)[:, -1:]
        acc = np.zeros((S, D), f32)
        for k in range(S):
            acc = acc + e[:, k:k + 1] * V[h, k][None, :]
        O[h] = acc / total
    return O


def np_cpu_rmsnorm(x, w, rows, dim, eps):
    """The reference test suite's CPU RMSNorm (test/mesh_encoder_test.c3:81-92):
    squares summed in order, inv_rms = 1 / sqrt(squares / dim + eps),
    out = x * inv_rms * w."""
    x = x.reshape(rows, dim)
    sq = np.add.accumulate(x * x, axis=1, dtype=f32)[:, -1:]
    inv = f32(1.0) / np.sqrt(sq / f32(dim) + f32(eps), dtype=f32)
    return (x * inv * w[None, :]).astype(f32)


def np_vae(Q, K, V, D, H, S, scale):
    """diffusion.slang:1846-1975 on [S, H*D] (head h at columns h*D..): keys in
    4096-key tiles with a running max / sum; per tile the scores are
    (q . k) * scale summed over d in order, the max and the exponential sum
    are 256 lane partials (lane g takes keys g, g+256, ...) folded by a
    halving tree, and the output gains sum_i p_i v_i over i in order after a
    rescale by exp(old_max - new_max). All queries of a head at once."""
    TILE = 4096
    O = np.zeros((S, H * D), f32)
    for h in range(H):
        q = Q[:, h * D:(h + 1) * D]
        k = K[:, h * D:(h + 1) * D]
        v = V[:, h * D:(h + 1) * D]
        acc = np.zeros((S, D), f32)
        run_max = np.full((S, 1), -1.0e30, f32)
        run_sum = np.zeros((S, 1), f32)
        for t0 in range(0, S, TILE):
            n = min(TILE, S - t0)
            dot = np.zeros((S, n), f32)
            for d in range(D):
                dot = dot + q[:, d:d + 1] * k[t0:t0 + n, d][None, :]
            sc = dot * f32(scale)
            tmax = sc.max(axis=1, keepdims=True)
            new_max = np.maximum(run_max, tmax)
            alpha = np.exp(run_max - new_max, dtype=f32)
            ev = np.exp(sc - new_max, dtype=f32)
            part = np.zeros((S, 256), f32)
            for c0 in range(0, n, 256):
                m = min(256, n - c0)
                part[:, :m] = part[:, :m] + ev[:, c0:c0 + m]
            w = 128
            while w > 0:
                part[:, :w] = part[:, :w] + part[:, w:2 * w]
                w //= 2
            vacc = np.zeros((S, D), f32)
            for i in range(n):
                vacc = vacc + ev[:, i:i + 1] * v[t0 + i][None, :]
            acc = acc * alpha + vacc
            run_sum = run_sum * alpha + part[:, :1]
            run_max = new_max
        O[:, h * D:(h + 1) * D] = acc * (f32(1.0) / run_sum)
    return O


def main():
    rng = np.random.default_rng(23)
    man = {}

    # batch_head_norm
    S, H, D = 5, 3, 128
    x = rng.standard_normal((S, H * D), dtype=f32)
    g = rng.uniform(0.8, 1.2, D).astype(f32)
    man["head_norm"] = {"params": {"S": S, "H": H, "D": D, "eps": 1e-5},
                        "x": save("head_norm_x", x), "gain": save("head_norm_gain", g),
                        "out": save("head_norm_out", np_head_norm(x, g, H, D, S, 1e-5))}

    # transpose_heads
    S, H, D = 7, 3, 8
    x = rng.standard_normal((S * H * D,), dtype=f32)
    man["transpose"] = {"params": {"S": S, "H": H, "D": D}, "x": save("transpose_x", x),
                        "out0": save("transpose_out0", np_transpose(x, S, H, D, 0)),
                        "out1": save("transpose_out1", np_transpose(x, S, H, D, 1))}

    # RoPE tables (Flux.1 style ids, Flux.2 4-axis, Z-Image axes)
    ids = np.zeros((3 + 6, 3), np.int32)
    ids[3:, 1] = np.repeat(np.arange(2), 3)
    ids[3:, 2] = np.tile(np.arange(3), 2)
    ids4 = np.zeros((9, 4), np.int32)
    ids4[:3, 3] = np.arange(3)
    ids4[3:, 1] = ids[3:, 1]
    ids4[3:, 2] = ids[3:, 2]
    idz = ids.copy()
    idz[:3, 0] = np.arange(1, 4)
    tabs = {}
    for name, pos, axes, theta in (("rope_flux1", ids, (16, 56, 56), 10000.0),
                                   ("rope_flux2", ids4, (32, 32, 32, 32), 2000.0),
                                   ("rope_zimage", idz, (32, 48, 48), 256.0)):
        c, s = np_tables(pos, axes, theta)
        tabs[name] = (c, s)
        man[name] = {"params": {"axes": list(axes), "theta": theta},
                     "pos": save(name + "_pos", pos.astype(f32)),
                     "cos": save(name + "_cos", c), "sin": save(name + "_sin", s)}

    # mrope on [H, S, 128] with the flux1 tables
    c, s = tabs["rope_flux1"]
    S, H = c.shape[0], 2
    x = rng.standard_normal((H, S, 128), dtype=f32)
    man["mrope"] = {"params": {"S": S, "H": H}, "x": save("mrope_x", x),
                    "cos": save("mrope_cos", c), "sin": save("mrope_sin", s),
                    "out": save("mrope_out", np_mrope(x, c, s, S, H))}

    # flash_attention_v2: ragged S = 45 (3 query blocks, 2 key blocks, tail 13)
    H, S, D = 2, 45, 128
    q = rng.standard_normal((H, S, D), dtype=f32)
    k = rng.standard_normal((H, S, D), dtype=f32)
    v = rng.standard_normal((H, S, D), dtype=f32)
    sc = 1.0 / np.sqrt(128.0)
    man["fa2"] = {"params": {"H": H, "S": S, "D": D, "scale": float(f32(sc))},
                  "q": save("fa2_q", q), "k": save("fa2_k", k), "v": save("fa2_v", v),
                  "out": save("fa2_out", np_fa2(q, k, v, D, H, S, f32(sc)))}

    # spatial_attention: D = 64, S = 37
    H, S, D = 2, 37, 64
    q = rng.standard_normal((H, S, D), dtype=f32)
    k = rng.standard_normal((H, S, D), dtype=f32)
    v = rng.standard_normal((H, S, D), dtype=f32)
    man["spatial"] = {"params": {"H": H, "S": S, "D": D, "scale": 0.125},
                      "q": save("spatial_q", q), "k": save("spatial_k", k),
                      "v": save("spatial_v", v),
                      "out": save("spatial_out", np_spatial(q, k, v, D, H, S, f32(0.125)))}

    # split_qkv
    n, dim = 5, 12
    qkv = rng.standard_normal((n, 3 * dim), dtype=f32)
    man["split_qkv"] = {"params": {"n_rows": n, "dim": dim}, "qkv": save("split_qkv_in", qkv),
                        "q": save("split_qkv_q", qkv[:, :dim]),
                        "k": save("split_qkv_k", qkv[:, dim:2 * dim]),
                        "v": save("split_qkv_v", qkv[:, 2 * dim:])}

    # Flux-style block: txt/img gains split at row 3, RoPE, fa2
    S, H, D = 9, 2, 128
    c, s = tabs["rope_flux1"]
    q = rng.standard_normal((S, H * D), dtype=f32)
    k = rng.standard_normal((S, H * D), dtype=f32)
    v = rng.standard_normal((S, H * D), dtype=f32)
    qg = rng.uniform(0.8, 1.2, (2, D)).astype(f32)
    kg = rng.uniform(0.8, 1.2, (2, D)).astype(f32)
    split = 3
    qn = np.concatenate([np_head_norm(q[:split], qg[0], H, D, split, 1e-6),
                         np_head_norm(q[split:], qg[1], H, D, S - split, 1e-6)])
    kn = np.concatenate([np_head_norm(k[:split], kg[0], H, D, split, 1e-6),
                         np_head_norm(k[split:], kg[1], H, D, S - split, 1e-6)])
    qt = np_mrope(np_transpose(qn, S, H, D, 0), c, s, S, H)
    kt = np_mrope(np_transpose(kn, S, H, D, 0), c, s, S, H)
    vt = np_transpose(v, S, H, D, 0)
    man["block_flux"] = {"params": {"S": S, "H": H, "D": D, "eps": 1e-6, "split": split,
                                    "scale": float(f32(1.0 / np.sqrt(128.0)))},
                         "q": save("block_q", q), "k": save("block_k", k),
                         "v": save("block_v", v), "q_gain": save("block_qg", qg),
                         "k_gain": save("block_kg", kg), "cos": save("block_cos", c),
                         "sin": save("block_sin", s),
                         "out": save("block_out", np_fa2(qt, kt, vt, D, H, S,
                                                         f32(1.0 / np.sqrt(128.0))))}

    # vae_attention: [S, H*D], two heads, S = 4100 crosses the 4096-key tile
    S, H, D = 4100, 2, 4
    q = rng.standard_normal((S, H * D), dtype=f32)
    k = rng.standard_normal((S, H * D), dtype=f32)
    v = rng.standard_normal((S, H * D), dtype=f32)
    sc = f32(0.5)
    man["vae"] = {"params": {"S": S, "H": H, "D": D, "scale": float(sc)},
                  "q": save("vae_q", q), "k": save("vae_k", k), "v": save("vae_v", v),
                  "out": save("vae_out", np_vae(q, k, v, D, H, S, sc))}

    # The reference test's cpu_attention on the spatial_attention and
    # flash_attention_v2 fixtures' inputs (no new random draws).
    for key in ("spatial", "fa2"):
        m = man[key]
        p = m["params"]
        ins = [np.fromfile(os.path.join(HERE, m[t]["file"]), dtype=f32, offset=16).reshape(
            m[t]["shape"]) for t in ("q", "k", "v")]
        man["cpu_attention_" + key] = {
            "params": p, "inputs_of": key,
            "out": save("cpu_attention_" + key + "_out",
                        np_cpu_attention(*ins, p["D"], p["H"], p["S"], f32(p["scale"])))}

    # The reference test's cpu_rmsnorm on the head_norm fixture: rows are
    # (token, head) pairs of D elements.
    m = man["head_norm"]
    p = m["params"]
    x = np.fromfile(os.path.join(HERE, m["x"]["file"]), dtype=f32, offset=16)
    g = np.fromfile(os.path.join(HERE, m["gain"]["file"]), dtype=f32, offset=16)
    man["cpu_rmsnorm_head_norm"] = {
        "params": p, "inputs_of": "head_norm",
        "out": save("cpu_rmsnorm_head_norm_out",
                    np_cpu_rmsnorm(x, g, p["S"] * p["H"], p["D"], p["eps"]).reshape(
                        p["S"], p["H"] * p["D"]))}

    with open(os.path.join(HERE, "manifest.json"), "w") as fh:
        json.dump(man, fh, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
