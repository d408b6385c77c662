"""CPU: pieces of bench.py that must hold without a GPU.

* The reference arm runs only the oracle: it loads the configurations'
  numpy recipe by path and never imports the product package (which maps
  the CUDA library).
* The float64 row-window restatement the multi-GPU strong-scaling block
  checks its outputs against agrees with the oracle's restatement of the
  reference block on a small case.
"""
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_does_not_load_the_product_library():
    code = (
        "import argparse, sys\n"
        "sys.argv = ['bench.py']\n"
        "import bench\n"
        "bench.run_reference(argparse.Namespace(config='plumbing', steps=1, warmup=0, gpus=1))\n"
        "assert 'llmr_attn' not in sys.modules, 'product package imported'\n"
        "maps = open('/proc/self/maps').read()\n"
        "assert 'libllmr_attn' not in maps, 'product library mapped'\n"
        "assert 'liboracle_attn' in maps\n")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    assert '"impl": "reference"' in out.stdout


def test_f64_rows_matches_oracle_block():
    import torch
    sys.path.insert(0, ROOT)
    sys.argv = ["bench.py"]
    import bench
    import oracle as O
    C = bench.configs_module()
    case = C.C3
    S, H, D = 300, 2, 128
    prep = C.prepare(case, O.rope_tables, seq_len=S, n_heads=H)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    q, k, v = (t(a).to(torch.bfloat16) for a in (prep.q, prep.k, prep.v))
    qg, kg, cos, sin = t(prep.q_gain), t(prep.k_gain), t(prep.cos), t(prep.sin)
    case_s = C.AttnCase(**{**case.__dict__, "seq_len": S, "n_heads": H, "split_row": 100})
    got = bench.f64_rows(q, k, v, qg, kg, cos, sin, case_s, range(90, 130), range(H)).numpy()
    want = O.attention_block(prep.q[0], prep.k[0], prep.v[0], H, D, case.scale, eps=case.eps,
                             q_gain=prep.q_gain, k_gain=prep.k_gain, split_row=100,
                             cos=prep.cos, sin=prep.sin)[90:130]
    err = np.abs(got - want)
    assert err.max() <= 1e-3 and err.mean() <= 5e-5, (err.max(), err.mean())
