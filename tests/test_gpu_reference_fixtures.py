"""GPU checks against fixtures produced by the reference's own Python code.

tests/golden/make_golden.py drove the reference's BatchQuantizedKVCache
(mlx_quantized_extensions.py) and its patched quantized SDPA (mlx_fused_attention.py)
on seeded inputs (over a NumPy stand-in for mlx).  Here the same inputs go through this
package's CUDA-backed caches and attention op:

* cache lifecycle (merge, update_and_fetch, make_mask, extend, filter, extract, trim,
  capacity growth): every Q4 tensor, offset, left padding, _idx and capacity identical;
* SDPA: within 2e-3 + 1e-3*|ref| of the reference's outputs (which round scores and
  probabilities to fp16; the kernels accumulate in fp32).
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import assert_close, pkg

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).parent / "golden"


def _bits(t):
    a = t.detach().cpu()
    return a.numpy().view(np.uint32) if a.dtype == torch.int32 else a.view(torch.int16).numpy().view(np.uint16)


def test_cache_lifecycle_matches_reference(cuda):
    f = np.load(GOLDEN / "ref_cache_lifecycle.npz")
    meta = {m["tag"]: m for m in json.loads(str(f["meta"]))}

    def inp(name):
        k = torch.from_numpy(f[f"in_{name}_k"].view(np.float16).copy()).to(cuda)
        v = torch.from_numpy(f[f"in_{name}_v"].view(np.float16).copy()).to(cuda)
        return k, v

    def check(tag, c):
        m = meta[tag]
        assert c._idx == m["idx"], tag
        assert c.offset.tolist() == m["offset"], tag
        assert c.left_padding.tolist() == m["left_padding"], tag
        if m["capacity"] is not None:
            assert c.keys[0].shape[-2] == m["capacity"], tag
            k, v = c.state[0], c.state[1]
            for nm, q in (("k", k), ("v", v)):
                for part, t in zip("csb", q):
                    np.testing.assert_array_equal(_bits(t), f[f"{tag}_{nm}{part}"], err_msg=f"{tag} {nm}{part}")

    c1 = pkg.QuantizedKVCache(group_size=64, bits=4)
    c1.update_and_fetch(*inp("c1"))
    c2 = pkg.QuantizedKVCache(group_size=64, bits=4)
    c2.update_and_fetch(*inp("c2"))
    batch = pkg.BatchQuantizedKVCache.merge([c1, c2])
    check("merge", batch)
    assert np.array_equal(batch.make_mask(1).to_dense().cpu().numpy(), f["mask_after_merge"])
    batch.update_and_fetch(*inp("u1"))
    check("update1", batch)
    assert np.array_equal(batch.make_mask(3, window_size=6).to_dense().cpu().numpy(), f["mask_window"])
    batch.update_and_fetch(*inp("u2"))
    check("update2", batch)
    c4 = pkg.QuantizedKVCache(group_size=64, bits=4)
    c4.update_and_fetch(*inp("c4"))
    other = pkg.BatchQuantizedKVCache.merge([c4])
    check("other", other)
    batch.extend(other)
    check("extend", batch)
    batch.filter([0, 2])
    check("filter", batch)
    e = batch.extract(1)
    assert e.offset == meta["extract"]["offset"]
    for nm, q in (("k", e.keys), ("v", e.values)):
        for part, t in zip("csb", q):
            np.testing.assert_array_equal(_bits(t), f[f"extract_{nm}{part}"])
    batch.trim(2)
    check("trim", batch)
    batch.update_and_fetch(*inp("u3"))
    check("update3", batch)


@pytest.mark.parametrize("name", sorted(p.stem[len("ref_sdpa_"):] for p in GOLDEN.glob("ref_sdpa_*.npz")))
def test_sdpa_matches_reference(cuda, name):
    f = np.load(GOLDEN / f"ref_sdpa_{name}.npz")
    q = torch.from_numpy(f["q"].view(np.float16).copy()).to(cuda)
    kq = (torch.from_numpy(f["kc"].view(np.int32).copy()).to(cuda),
          torch.from_numpy(f["ks"].view(np.float16).copy()).to(cuda),
          torch.from_numpy(f["kb"].view(np.float16).copy()).to(cuda))
    vq = (torch.from_numpy(f["vc"].view(np.int32).copy()).to(cuda),
          torch.from_numpy(f["vs"].view(np.float16).copy()).to(cuda),
          torch.from_numpy(f["vb"].view(np.float16).copy()).to(cuda))
    mask = None
    if "mask_str" in f.files:
        mask = str(f["mask_str"])
    elif "mask" in f.files:
        m = f["mask"]
        mask = torch.from_numpy(m.copy()).to(cuda)
    out = pkg.quantized_scaled_dot_product_attention(q, kq, vq, float(f["scale"]), mask)
    ref = f["out"].view(np.float16).astype(np.float32)
    assert_close(out.float().cpu().numpy(), ref, what=f"reference sdpa {name}")
