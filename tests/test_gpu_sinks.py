"""Attention sinks over a Q4 cache (GPT-OSS geometry: head_dim 64, n_rep 8, 128-token
sliding windows), on the decode, split-KV combine and tcgen05 prefill paths.

The reference dequantizes the Q4 tuples to fp16 and calls the fast SDPA with the sink
logits (mlx_sink_compat.py:46-69); the kernels here fold the sinks into the softmax
normaliser and read the Q4 blocks directly.  Tolerance: |gpu - oracle| <= 2e-3 +
1e-3 * |oracle| (fp32 accumulation; fp32 outputs where the output dtype would add its own
rounding).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import assert_close, pkg

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("merge_mode")]

GOLDEN = Path(__file__).parent / "golden"
F16 = 0


def _bits(t):
    a = t.detach().cpu()
    return a.numpy().view(np.uint32) if a.dtype == torch.int32 else a.view(torch.int16).numpy().view(np.uint16)


class _Q4Cache:
    bits = 4
    group_size = 64


def _case(B, Hq, Hkv, N, D, L, seed, cuda, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, D, generator=g).to(dtype)
    q = torch.randn(B, Hq, L, D, generator=g).to(dtype)
    sinks = torch.randn(Hq, generator=g) * 2 + 6  # comparable to the mass of thousands of keys
    return q, pkg.quantize(k.to(cuda)), pkg.quantize(v.to(cuda)), sinks


def _oracle(orc, q, kq, vq, scale, sinks, **kw):
    return orc.attention(q.float().numpy(), tuple(_bits(t) for t in kq), tuple(_bits(t) for t in vq),
                         scale, sdtype=F16, sinks=sinks.numpy(), **kw)


@pytest.mark.parametrize("name", sorted(p.stem[len("ref_sinks_"):] for p in GOLDEN.glob("ref_sinks_*.npz")))
def test_sinks_match_reference_shim(cuda, name):
    """Outputs of the reference's own sink shim (tests/golden/make_golden.py)."""
    f = np.load(GOLDEN / f"ref_sinks_{name}.npz")
    q = torch.from_numpy(f["q"].view(np.float16).copy()).to(cuda)
    kq = tuple(torch.from_numpy(f[n].view(np.int32 if n.endswith("c") else np.float16).copy()).to(cuda)
               for n in ("kc", "ks", "kb"))
    vq = tuple(torch.from_numpy(f[n].view(np.int32 if n.endswith("c") else np.float16).copy()).to(cuda)
               for n in ("vc", "vs", "vb"))
    mask = None
    if "mask_str" in f.files:
        mask = str(f["mask_str"])
    elif "mask" in f.files:
        mask = torch.from_numpy(f["mask"].copy()).to(cuda)
    sinks = torch.from_numpy(f["sinks"].copy()).to(cuda)
    out = pkg.scaled_dot_product_attention(q, kq, vq, _Q4Cache(), float(f["scale"]), mask, sinks=sinks)
    ref = f["out"].view(np.float16).astype(np.float32)
    assert_close(out.float().cpu().numpy(), ref, what=f"reference sink shim {name}")


@pytest.mark.parametrize("N,window", [(1000, 0), (1000, 128), (6000, 0), (6000, 128)])
def test_decode_sinks_gpt_oss_geometry(cuda, orc, N, window):
    """Decode over 64 query / 8 KV heads of dim 64, full and sliding-window layers; N=6000
    splits each sequence into several chunks, so the sinks go through the combine kernel."""
    B, Hq, Hkv, D = 2, 64, 8, 64
    q, kq, vq, sinks = _case(B, Hq, Hkv, N, D, 1, seed=N + window, cuda=cuda)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), n, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), 0.125, kv_len, n, causal=True, window=window,
                                out_dtype=torch.float32, mode="decode", sinks=sinks.to(cuda))
    want = _oracle(orc, q, kq, vq, 0.125, sinks, causal=True, window=window)
    assert_close(got.cpu().numpy(), want, what=f"decode sinks N={N} window={window}")
    # the sinks' effect is reproduced (guards against the argument being dropped)
    plain = pkg.kernels.attention(view, q.to(cuda), 0.125, kv_len, n, causal=True, window=window,
                                  out_dtype=torch.float32, mode="decode")
    effect = np.abs(want - orc.attention(q.float().numpy(), tuple(_bits(t) for t in kq),
                                         tuple(_bits(t) for t in vq), 0.125, sdtype=F16,
                                         causal=True, window=window)).max()
    assert effect > 1e-3
    assert (plain - got).abs().max().item() > 0.5 * effect


def test_prefill_sinks(cuda, orc):
    """A 256-token causal chunk over a 700-token prefix on the tcgen05 prefill kernel."""
    B, Hq, Hkv, D, P, L = 1, 16, 2, 64, 700, 256
    q, kq, vq, sinks = _case(B, Hq, Hkv, P + L, D, L, seed=3, cuda=cuda)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), n, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), 0.125, kv_len, n, causal=True,
                                out_dtype=torch.float32, mode="prefill", sinks=sinks.to(cuda))
    want = _oracle(orc, q, kq, vq, 0.125, sinks, causal=True)
    assert_close(got.cpu().numpy(), want, what="prefill sinks")


def test_sinks_fully_masked_row_is_zero(cuda, orc):
    """With every key masked the sink takes all the weight and the output is zero."""
    q, kq, vq, sinks = _case(1, 8, 1, 40, 64, 1, seed=5, cuda=cuda)
    keep = torch.zeros(1, 1, 1, 40, dtype=torch.bool)
    got = pkg.scaled_dot_product_attention(q.to(cuda), kq, vq, _Q4Cache(), 0.125, keep.to(cuda),
                                           sinks=sinks.to(cuda))
    want = _oracle(orc, q, kq, vq, 0.125, sinks, causal=False, mask=keep.numpy().astype(np.float32),
                   mask_kind=1)
    assert np.abs(want).max() == 0.0
    assert_close(got.float().cpu().numpy(), want, what="fully masked with sinks")
