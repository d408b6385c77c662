"""Shared test setup: import paths, the `gpu` marker, golden-vector loading."""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("", "llm-runner_b200", "oracle"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")
HEADER = b"C3_DEBUG_TENSOR\x00"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def load_golden(entry):
    """Reads one fixture in the reference's dump format (test/README.md:64-68)."""
    with open(os.path.join(GOLDEN, entry["file"]), "rb") as fh:
        raw = fh.read()
    assert raw[:16] == HEADER
    return np.frombuffer(raw[16:], dtype=np.float32).reshape(entry["shape"]).copy()


@pytest.fixture(scope="session")
def manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as fh:
        return json.load(fh)


@pytest.fixture(scope="session")
def ctx():
    """A library context on cuda:0 (GPU tests only)."""
    import torch
    import llmr_attn
    torch.cuda.init()
    c = llmr_attn.Context(0, workspace_bytes=0)
    yield c
    c.close()
