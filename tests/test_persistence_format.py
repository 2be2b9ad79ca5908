"""Q4 cache file format (CPU): the files persistence.save_blocks writes are standard
safetensors files with the reference's tensor names, shapes and dtypes
(safetensors_cache_adapter.py:141-199, :284-327), checked with the independent
safetensors reader; read_header parses files the safetensors writer produced."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import pkg

safetensors = pytest.importorskip("safetensors")
from safetensors.numpy import save_file  # noqa: E402
from safetensors import safe_open  # noqa: E402

persistence = __import__(pkg.__name__ + ".persistence", fromlist=["persistence"])


def fake_pool(H=2, kd=128, vd=64, bt=256, dtype=torch.float16):
    return SimpleNamespace(n_kv_heads=H, k_dim=kd, v_dim=vd, block_tokens=bt, dtype=dtype)


def test_layout_names_shapes_offsets():
    pool = fake_pool()
    header, ids, toks, offs, nbytes = persistence.block_layout(pool, {0: [(5, 256), (9, 44)],
                                                                      3: [(1, 256)]})
    assert ids == [5, 9, 1] and toks == [256, 44, 256]
    assert header["L0_B1_K_weights"] == {"dtype": "U32", "shape": [1, 2, 44, 16],
                                         "data_offsets": header["L0_B1_K_weights"]["data_offsets"]}
    assert header["L3_B0_V_scales"]["shape"] == [1, 2, 256, 1]
    assert header["L3_B0_V_scales"]["dtype"] == "F16"
    # tensors tile the data section without gaps, in the packing order
    spans = sorted(e["data_offsets"] for e in header.values())
    assert spans[0][0] == 0 and spans[-1][1] == nbytes
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert [o[0] for o in offs] == [header[f"L{l}_B{b}_K_weights"]["data_offsets"][0]
                                    for l, b in [(0, 0), (0, 1), (3, 0)]]


def test_written_file_reads_with_safetensors(tmp_path):
    pool = fake_pool(H=2, kd=64, vd=64, bt=32)
    layers = {0: [(0, 32), (1, 7)], 1: [(2, 32)]}
    header, _, _, _, nbytes = persistence.block_layout(pool, layers)
    data = np.random.default_rng(0).integers(0, 256, nbytes, dtype=np.uint8)
    path = tmp_path / "agent.safetensors"
    with path.open("wb") as f:
        f.write(persistence._encode_header(header, {"block_tokens": 32, "n_layers": 2}))
        f.write(data.tobytes())
    with safe_open(str(path), framework="numpy") as f:
        assert f.metadata() == {"block_tokens": "32", "n_layers": "2"}
        assert sorted(f.keys()) == sorted(header)
        for name, e in header.items():
            t = f.get_tensor(name)
            assert list(t.shape) == e["shape"]
            assert t.dtype == (np.uint32 if e["dtype"] == "U32" else np.float16)
            s0, s1 = e["data_offsets"]
            assert t.tobytes() == data[s0:s1].tobytes()


def test_read_header_of_safetensors_written_file(tmp_path):
    rng = np.random.default_rng(1)
    tensors = {"L0_B0_K_weights": rng.integers(0, 2**32, (1, 2, 10, 16), dtype=np.uint32),
               "L0_B0_K_scales": rng.standard_normal((1, 2, 10, 2)).astype(np.float16)}
    path = tmp_path / "ref.safetensors"
    save_file(tensors, str(path), metadata={"model_id": "x"})
    header, meta, start = persistence.read_header(path)
    assert meta == {"model_id": "x"}
    raw = path.read_bytes()[start:]
    for name, arr in tensors.items():
        s0, s1 = header[name]["data_offsets"]
        assert raw[s0:s1] == arr.tobytes()
        assert header[name]["shape"] == list(arr.shape)


def test_agent_id_validation(tmp_path):
    store = persistence.SafetensorsQ4Store.__new__(persistence.SafetensorsQ4Store)
    for bad in ["", "a/b", "../x", "x" * 257, "a b"]:
        with pytest.raises(persistence.CachePersistenceError):
            store._validate_agent_id(bad)
    store._validate_agent_id("agent_1-A")
