"""am_q4_decode_noalloc: split-KV decode for callers that cannot allocate device memory.

Such callers (a serving loop with a fixed, pre-planned memory budget, a host runtime
without its own CUDA allocator, a binding that only passes plain pointers) get the same
decode kernel with its scratch taken from a 16 MiB array compiled into the library.  This
file checks, through the C ABI, that two calls in a row give the same outputs as
am_q4_decode with a caller-provided workspace (within the attention tolerance), and that
calls needing more than the static scratch are rejected.  It is named so pytest collects
it last and passes both alone and after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_close, pkg

pytestmark = pytest.mark.gpu


def _args(view, q, out, kv_len, max_len, scale):
    a = pkg._lib.AttnArgs()
    a.q = q.data_ptr()
    a.q_dtype = pkg._lib.DTYPE_F16
    a.batch, a.n_q_heads, a.q_len = q.shape[0], q.shape[1], q.shape[2]
    a.q_stride_b, a.q_stride_h, a.q_stride_l = q.stride(0), q.stride(1), q.stride(2)
    a.out = out.data_ptr()
    a.out_dtype = pkg._lib.DTYPE_F32
    a.o_stride_b, a.o_stride_h, a.o_stride_l = out.stride(0), out.stride(1), out.stride(2)
    a.scale = scale
    a.kv_len = kv_len.data_ptr()
    a.kv_start = None
    a.max_kv_len = max_len
    a.mask_kind = pkg._lib.MASK_NONE
    return a


def _case(cuda, seed, B=3, Hq=32, Hkv=8, N=3000, D=128):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, Hkv, N, D, generator=g).half().to(cuda)
    v = torch.randn(B, Hkv, N, D, generator=g).half().to(cuda)
    q = torch.randn(B, Hq, 1, D, generator=g).half().to(cuda)
    view, n = pkg.kernels.contiguous_view(pkg.quantize(k), pkg.quantize(v))
    kv_len = torch.full((B,), n, dtype=torch.int32, device=cuda)
    return view, q, kv_len, n


def test_noalloc_decode_matches_workspace_decode_twice(cuda, merge_mode):
    lib = pkg._lib.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call, seed in enumerate((1, 2)):
        view, q, kv_len, n = _case(cuda, seed)
        ref = torch.empty(q.shape[0], q.shape[1], 1, 128, dtype=torch.float32, device=cuda)
        got = torch.empty_like(ref)
        a_ref = _args(view, q, ref, kv_len, n, 128 ** -0.5)
        need = lib.am_q4_attention_workspace_bytes(ctypes.byref(view.desc), ctypes.byref(a_ref))
        if merge_mode == "workspace":  # the split path through the scratch is exercised
            assert 0 < need <= pkg._lib.STATIC_DECODE_SCRATCH_BYTES
        else:  # split chunks merge inside a cluster: no scratch at all
            assert need == 0
        ws = torch.empty(max(need, 16), dtype=torch.uint8, device=cuda)
        rc = lib.am_q4_decode(ctypes.byref(view.desc), ctypes.byref(a_ref), ws.data_ptr(), need, stream)
        assert rc == 0, lib.am_last_error()
        a_got = _args(view, q, got, kv_len, n, 128 ** -0.5)
        rc = lib.am_q4_decode_noalloc(ctypes.byref(view.desc), ctypes.byref(a_got), stream)
        assert rc == 0, lib.am_last_error()
        torch.cuda.synchronize(cuda)
        assert_close(got.cpu().numpy(), ref.cpu().numpy(), what=f"noalloc call {call}")


def test_noalloc_rejects_requests_beyond_the_static_scratch(cuda):
    lib = pkg._lib.load()
    view, q, kv_len, n = _case(cuda, 3, B=2, N=64)
    out = torch.empty(2, 32, 1, 128, dtype=torch.float32, device=cuda)
    a = _args(view, q, out, kv_len, 1 << 24, 0.1)  # claims 16M-token contexts
    a.batch = 2
    need = lib.am_q4_attention_workspace_bytes(ctypes.byref(view.desc), ctypes.byref(a))
    assert need > pkg._lib.STATIC_DECODE_SCRATCH_BYTES
    rc = lib.am_q4_decode_noalloc(ctypes.byref(view.desc), ctypes.byref(a), None)
    assert rc == pkg._lib.AM_ERR_WORKSPACE
    assert b"static scratch" in lib.am_last_error()


def test_noalloc_paged_bf16_through_static_scratch(cuda, monkeypatch):
    """Paged layout with bf16 scales, split chunks merged through the scratch (cluster merging
    off): two calls in a row agree with am_q4_decode given a caller workspace."""
    monkeypatch.setenv("AM_Q4_DECODE_MAX_CLUSTER", "0")
    lib = pkg._lib.load()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    Hq, Hkv, D, bt = 16, 4, 128, 256
    lens = [3000, 700, 5000]
    nb = sum(-(-n // bt) for n in lens)
    pool = pkg.PagedQ4Pool(Hkv, D, D, nb, bt, torch.bfloat16, cuda)
    g = torch.Generator().manual_seed(9)
    perm = torch.randperm(nb, generator=g)
    table = torch.full((len(lens), max(-(-n // bt) for n in lens)), -1, dtype=torch.int32)
    used = 0
    for a, n in enumerate(lens):
        k = -(-n // bt)
        table[a, :k] = perm[used:used + k]
        used += k
    tab = table.to(cuda)
    for a, n in enumerate(lens):
        kk = torch.randn(1, Hkv, n, D, generator=g).bfloat16().to(cuda)
        vv = torch.randn(1, Hkv, n, D, generator=g).bfloat16().to(cuda)
        pkg.kernels.append(pool.view(tab[a:a + 1].contiguous()), kk, vv,
                           torch.zeros(1, dtype=torch.int32, device=cuda))
    view = pool.view(tab)
    kv_len = torch.tensor(lens, dtype=torch.int32, device=cuda)
    for call in range(2):
        q = torch.randn(len(lens), Hq, 1, D, generator=g).half().to(cuda)
        ref = torch.empty(len(lens), Hq, 1, D, dtype=torch.float32, device=cuda)
        got = torch.empty_like(ref)
        a_ref = _args(view, q, ref, kv_len, max(lens), D ** -0.5)
        need = lib.am_q4_attention_workspace_bytes(ctypes.byref(view.desc), ctypes.byref(a_ref))
        assert 0 < need <= pkg._lib.STATIC_DECODE_SCRATCH_BYTES
        ws = torch.empty(need, dtype=torch.uint8, device=cuda)
        rc = lib.am_q4_decode(ctypes.byref(view.desc), ctypes.byref(a_ref), ws.data_ptr(), need, stream)
        assert rc == 0, lib.am_last_error()
        a_got = _args(view, q, got, kv_len, max(lens), D ** -0.5)
        rc = lib.am_q4_decode_noalloc(ctypes.byref(view.desc), ctypes.byref(a_got), stream)
        assert rc == 0, lib.am_last_error()
        torch.cuda.synchronize(cuda)
        assert_close(got.cpu().numpy(), ref.cpu().numpy(), what=f"paged bf16 noalloc call {call}")


def test_noalloc_reports_bad_sizes_as_invalid(cuda):
    """Negative sizes are argument errors (AM_ERR_INVALID), not scratch-size errors."""
    lib = pkg._lib.load()
    view, q, kv_len, n = _case(cuda, 4, B=1, N=64)
    out = torch.empty(1, 32, 1, 128, dtype=torch.float32, device=cuda)
    a = _args(view, q, out, kv_len, n, 0.1)
    a.max_kv_len = -5
    assert lib.am_q4_decode_noalloc(ctypes.byref(view.desc), ctypes.byref(a), None) == pkg._lib.AM_ERR_INVALID
    assert b"max_kv_len" in lib.am_last_error()
