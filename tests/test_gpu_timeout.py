"""The kernels' bounded waits give up cleanly (failure detection without a GPU fault).

AM_Q4_TEST_WAIT_LIMIT_NS=0 makes every pipeline wait inside the kernels give up at once, as
a wait whose phase never completes does when its limit runs out.  The kernel must then
flag AM_STATUS_TIMEOUT in the status word, let its copies in flight land, free what it
holds and return; the call returns to the host, the context stays usable, and the next
call with the normal limit is correct again.  Nothing here faults, traps or
hangs: the waits are bounded either way.
"""

import numpy as np
import pytest
import torch

from conftest import assert_close, pkg
from test_gpu_decode import _bits, make_case, oracle

pytestmark = pytest.mark.gpu

TIMEOUT = 4  # AM_STATUS_TIMEOUT


def _decode(cuda, q, kq, vq, status=None):
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((q.shape[0],), n, dtype=torch.int32, device=cuda)
    return pkg.kernels.attention(view, q.to(cuda), q.shape[-1] ** -0.5, kv_len, n,
                                 out_dtype=torch.float32, status=status, mode="decode")


@pytest.mark.usefixtures("merge_mode")
def test_decode_wait_timeout_is_flagged_and_recovers(cuda, orc, monkeypatch):
    q, kq, vq = make_case(2, 32, 8, 3000, 128, 128, cuda=cuda, seed=21)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    monkeypatch.setenv("AM_Q4_TEST_WAIT_LIMIT_NS", "0")
    out = _decode(cuda, q, kq, vq, status)
    torch.cuda.synchronize(cuda)
    assert int(status.item()) & TIMEOUT, "a zero wait limit must trip the timeout path"
    assert out.shape == (2, 32, 1, 128)
    monkeypatch.delenv("AM_Q4_TEST_WAIT_LIMIT_NS")
    status.zero_()
    got = _decode(cuda, q, kq, vq, status)
    torch.cuda.synchronize(cuda)
    assert int(status.item()) == 0
    want = oracle(orc, q, kq, vq, 128 ** -0.5, causal=False)
    assert_close(got.cpu().numpy(), want, what="decode after a timed-out call")


def test_paged_decode_wait_timeout_is_flagged_and_recovers(cuda, orc, monkeypatch):
    """The paged layout (block table, 2-D tensor-map loads of scattered blocks)."""
    Hq, Hkv, D, bt, n = 16, 8, 128, 256, 1500
    pool = pkg.PagedQ4Pool(Hkv, D, D, 12, bt, torch.float16, cuda)
    g = torch.Generator().manual_seed(3)
    table = torch.randperm(12, generator=g)[:6].to(torch.int32).reshape(1, 6)
    tab = table.to(cuda)
    k = torch.randn(1, Hkv, n, D, generator=g).half()
    v = torch.randn(1, Hkv, n, D, generator=g).half()
    pkg.kernels.append(pool.view(tab), k.to(cuda), v.to(cuda), torch.zeros(1, dtype=torch.int32, device=cuda))
    q = torch.randn(1, Hq, 1, D, generator=g).half()
    kv_len = torch.tensor([n], dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    monkeypatch.setenv("AM_Q4_TEST_WAIT_LIMIT_NS", "0")
    pkg.kernels.attention(pool.view(tab), q.to(cuda), D ** -0.5, kv_len, n, status=status,
                          out_dtype=torch.float32, mode="decode")
    torch.cuda.synchronize(cuda)
    assert int(status.item()) & TIMEOUT
    monkeypatch.delenv("AM_Q4_TEST_WAIT_LIMIT_NS")
    status.zero_()
    got = pkg.kernels.attention(pool.view(tab), q.to(cuda), D ** -0.5, kv_len, n, status=status,
                                out_dtype=torch.float32, mode="decode")
    torch.cuda.synchronize(cuda)
    assert int(status.item()) == 0
    want = orc.attention(q.float().numpy(), tuple(_bits(t) for t in pool.k),
                         tuple(_bits(t) for t in pool.v), D ** -0.5, n_kv_heads=Hkv, layout=1,
                         block_table=table.numpy(), kv_len=np.array([n]), causal=False)
    assert_close(got.cpu().numpy(), want, what="paged decode after a timed-out call")


@pytest.mark.parametrize("geom", [(16, 4, 128, 128), (16, 16, 192, 128)], ids=["d128", "k192_v128"])
def test_prefill_wait_timeout_is_flagged_and_recovers(cuda, orc, monkeypatch, geom):
    """The tcgen05 prefill kernels (TMA-fed two-tile, and the one-tile kernel whose producer
    warps dequantize the tiles): producer, MMA issuer and softmax warps all give up, the
    kernel waits for its loads and MMAs in flight, frees its TMEM and returns; the next
    call (fresh TMEM allocations on every SM) is correct."""
    Hq, Hkv, D, Dv = geom
    B, L, N = 2, 256, 1200
    q, kq, vq = make_case(B, Hq, Hkv, N, D, Dv, L=L, cuda=cuda, seed=23)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), n, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    monkeypatch.setenv("AM_Q4_TEST_WAIT_LIMIT_NS", "0")
    pkg.kernels.attention(view, q.to(cuda), D ** -0.5, kv_len, n, causal=True, status=status,
                          out_dtype=torch.float32, mode="prefill")
    torch.cuda.synchronize(cuda)
    assert int(status.item()) & TIMEOUT
    monkeypatch.delenv("AM_Q4_TEST_WAIT_LIMIT_NS")
    status.zero_()
    got = pkg.kernels.attention(view, q.to(cuda), D ** -0.5, kv_len, n, causal=True, status=status,
                                out_dtype=torch.float32, mode="prefill")
    torch.cuda.synchronize(cuda)
    assert int(status.item()) == 0
    want = oracle(orc, q, kq, vq, D ** -0.5, causal=True)
    assert_close(got.cpu().numpy(), want, what="prefill after a timed-out call")
