"""Test configuration: the `gpu` marker, package import, shared helpers.

Tests marked ``gpu`` need a CUDA device (B200) and the built libamq4.so; everything else
runs on the CPU.  The oracle under oracle/ is the checker in both kinds of tests.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402

pkg = load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and libamq4.so")


@pytest.fixture(scope="session")
def am():
    return pkg


@pytest.fixture(scope="session")
def orc():
    from oracle import q4_oracle

    q4_oracle.build()
    return q4_oracle


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(params=["cluster", "workspace"])
def merge_mode(request, monkeypatch):
    """Split-KV decode merges the partials of a column's chunks either inside one
    thread-block cluster (the default where the chunks fit one cluster) or through the
    workspace and combine_kernel (AM_Q4_DECODE_MAX_CLUSTER=0); a test using this fixture
    runs once with each."""
    if request.param == "workspace":
        monkeypatch.setenv("AM_Q4_DECODE_MAX_CLUSTER", "0")
    else:
        monkeypatch.delenv("AM_Q4_DECODE_MAX_CLUSTER", raising=False)
    return request.param


def assert_close(got, want, atol=2e-3, rtol=1e-3, what=""):
    """The attention tolerance: |got - want| <= atol + rtol * |want| elementwise."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} of {err.size} elements out of tolerance; "
                             f"max err {err.max():.3e} at {i}: got {got[i]} want {want[i]}")


# Largest relative rounding error of storing a value in a 16-bit output dtype (half an ulp):
# fp16 keeps 11 significant bits, bf16 8.
OUT_ROUNDING = {"float16": 2.0 ** -11, "bfloat16": 2.0 ** -8, "float32": 0.0}


def assert_close_out(got, want, out_dtype, what=""):
    """The attention tolerance for outputs stored in a 16-bit dtype: the fp32 bound
    2e-3 + 1e-3 * |want| plus the dtype's own rounding of the result (half an ulp,
    OUT_ROUNDING relative).  Cases that check the kernel's arithmetic alone use fp32 outputs
    and assert_close."""
    name = str(out_dtype).replace("torch.", "")
    assert_close(got, want, atol=2e-3, rtol=1e-3 + OUT_ROUNDING[name], what=what)
