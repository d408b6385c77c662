"""CPU: the C-ABI library loads, exports every declared entry point, its host
logic matches the oracle, and it fails loudly without an sm_100 GPU."""
import ctypes
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "llmr_attn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(llmr_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    import llmr_attn
    names = declared_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", llmr_attn.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\s[TW]\s+(\S+)$", out, flags=re.M))
    missing = [n for n in names if n not in exported]
    assert not missing, missing


@pytest.mark.parametrize("py_name,c_name", [("AttnDesc", "llmr_attn_desc"),
                                             ("QkvDesc", "llmr_qkv_desc"),
                                             ("ProjDesc", "llmr_proj_desc"),
                                             ("IpcHandle", "llmr_ipc_handle")])
def test_desc_layout_matches_c(py_name, c_name):
    """The ctypes structs have the C structs' sizes and field offsets."""
    import llmr_attn
    cls = getattr(llmr_attn, py_name)
    fields = [f[0] for f in cls._fields_]
    src = '#include <stdio.h>\n#include <stddef.h>\n#include "' + HEADER + '"\nint main(){'
    src += 'printf("%zu\\n", sizeof(' + c_name + '));'
    for f in fields:
        src += 'printf("%zu\\n", offsetof(' + c_name + ', ' + f + '));'
    src += "return 0;}"
    with tempfile.TemporaryDirectory() as td:
        c = os.path.join(td, "t.c")
        exe = os.path.join(td, "t")
        open(c, "w").write(src)
        cc = "/usr/bin/gcc" if os.path.exists("/usr/bin/gcc") else "gcc"
        subprocess.run([cc, c, "-o", exe], check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True,
                                               check=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(cls)
    for f, off in zip(fields, vals[1:]):
        assert getattr(cls, f).offset == off, f


@pytest.mark.parametrize("axes,theta", [((16, 56, 56), 10000.0), ((32, 48, 48), 256.0),
                                        ((32, 32, 32, 32), 2000.0)])
def test_host_rope_tables_bit_exact_with_oracle(axes, theta):
    import llmr_attn
    import oracle as O
    from llmr_attn import configs
    ids = configs.flux_ids(7, 5, 6) if len(axes) == 3 else np.stack(
        [np.zeros(37), np.arange(37) // 6, np.arange(37) % 6, np.arange(37)], 1)
    ids = ids.astype(np.int32)
    c1, s1 = llmr_attn.rope_tables(ids, axes, theta)
    c2, s2 = O.rope_tables(ids, axes, theta)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(s1, s2)


def test_rope_tables_rejects_odd_axis():
    import llmr_attn
    with pytest.raises(llmr_attn.LlmrError):
        llmr_attn.rope_tables(np.zeros((2, 2), np.int32), (3, 5), 100.0)


def test_workspace_sizes():
    import llmr_attn as L
    cfg = L.AttnConfig(n_heads=24, head_dim=128, scale=0.088, norm_q=True, norm_k=True,
                       rope=True)
    d = L.make_desc(cfg, 1, 4608, L.BF16, L.BF16)
    assert L.workspace_bytes(d) == 3 * 24 * 4608 * 128 * 2
    raw = L.AttnConfig(n_heads=16, head_dim=64, scale=0.125)
    assert L.workspace_bytes(L.make_desc(raw, 1, 1370, L.F16, L.F16)) == 0
    ex = L.AttnConfig(n_heads=4, head_dim=64, scale=0.125, exact=True)
    # fp32 Q, K, V and, for the tensor-core path (D = 64), their TF32 residuals
    assert L.workspace_bytes(L.make_desc(ex, 1, 256, L.F32, L.F32)) == 9 * 4 * 256 * 64 * 4
    assert L.workspace_bytes(L.make_desc(ex, 1, 1370, L.F32, L.F32)) == \
        (7 * 4 * 1370 * 64 + 2 * 4 * 64 * 1372) * 4
    ex128 = L.AttnConfig(n_heads=4, head_dim=128, scale=0.088, exact=True)
    assert L.workspace_bytes(L.make_desc(ex128, 1, 256, L.F32, L.F32)) == 3 * 4 * 256 * 128 * 4
    vae = L.AttnConfig(n_heads=1, head_dim=512, scale=512 ** -0.5)
    assert L.workspace_bytes(L.make_desc(vae, 1, 16384, L.F32, L.F32)) == 3 * 16384 * 512 * 2
    assert L.workspace_bytes(L.make_desc(vae, 1, 16384, L.F16, L.F16)) == 0


def test_configs_flops_and_shapes():
    from llmr_attn import configs as C
    assert C.C3.flops == pytest.approx(2.609e11, rel=1e-3)
    assert C.C4.flops == pytest.approx(5.818e11, rel=1e-3)
    assert C.C5.flops == pytest.approx(1.403e13, rel=1e-3)
    assert C.case_ids(C.C3).shape == (4608, 3)
    assert C.case_ids(C.C4).shape == (4352, 3)
    assert C.case_ids(C.C5).shape == (33792, 3)
    q, k, v, qg, kg = C.make_inputs(C.C3, seq_len=40, n_heads=2)
    assert q.shape == (1, 40, 2, 128) and qg.shape == (2, 128)
    # values are bf16-representable
    assert np.array_equal(C.round_to(q, "bf16"), q)


def test_no_gpu_fails_loudly():
    """Without an sm_100 device the context cannot be created: no fallback."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import llmr_attn
    h = ctypes.c_void_p()
    rc = llmr_attn.lib.llmr_ctx_create(0, 0, None, ctypes.byref(h))
    assert rc == llmr_attn.ENODEV
