"""GPU parity of the split-KV decode kernel against the CPU oracle.

Tolerance (attention outputs): |gpu - oracle| <= 2e-3 + 1e-3 * |oracle|, fp32 accumulation.
Cases cover the geometries of the reference's tests and the benchmark configurations at
reduced sizes: Llama GQA 32/8 D128, Gemma 16/8 D256 with sliding windows, DeepSeek MLA
K192/V128 (n_rep 1), asymmetric K128/V64, D64; masks (none, causal string, boolean,
additive, structured left padding / window), bf16, paged vs contiguous, B=1 vs B=2.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_close, assert_close_out, pkg

# every case runs with both merges of split chunks (conftest.merge_mode)
pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("merge_mode")]

F16, BF16 = 0, 1


def _bits(t):
    a = t.detach().cpu()
    return a.numpy().view(np.uint32) if a.dtype == torch.int32 else a.view(torch.int16).numpy().view(np.uint16)


def make_case(B, Hq, Hkv, N, dk, dv, L=1, dtype=torch.float16, qdtype=None, seed=0, cuda=None):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, Hkv, N, dk, generator=g).to(dtype)
    v = torch.randn(B, Hkv, N, dv, generator=g).to(dtype)
    q = torch.randn(B, Hq, L, dk, generator=g).to(qdtype or dtype)
    kq = pkg.quantize(k.to(cuda))
    vq = pkg.quantize(v.to(cuda))
    return q, kq, vq


def oracle(orc, q, kq, vq, scale, **kw):
    sdt = BF16 if kq[1].dtype == torch.bfloat16 else F16
    return orc.attention(q.float().numpy(), tuple(_bits(t) for t in kq), tuple(_bits(t) for t in vq),
                         scale, sdtype=sdt, **kw)


GEOMS = [
    # (B, Hq, Hkv, N, dk, dv)
    (2, 32, 8, 2048, 128, 128),   # one Llama-3.1-8B layer at its benchmark shape
    (3, 16, 8, 777, 256, 256),    # Gemma-3 geometry
    (2, 16, 16, 1500, 192, 128),  # DeepSeek-V2 MLA (n_rep 1)
    (2, 8, 4, 333, 128, 64),      # asymmetric K/V
    (1, 4, 1, 100, 64, 64),       # small head dim, n_rep 4
    (2, 12, 4, 5, 128, 128),      # N < one tile
    (1, 4, 1, 40000, 64, 64),     # more chunks than one cluster holds: workspace + combine
]


@pytest.mark.parametrize("geom", GEOMS, ids=lambda g: "x".join(map(str, g)))
def test_decode_matches_oracle(cuda, orc, geom):
    B, Hq, Hkv, N, dk, dv = geom
    q, kq, vq = make_case(B, Hq, Hkv, N, dk, dv, cuda=cuda, seed=N)
    scale = dk ** -0.5
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, scale, None)
    assert got.dtype == q.dtype and got.shape == (B, Hq, 1, dv)
    want = oracle(orc, q, kq, vq, scale, causal=False)
    assert_close(got.float().cpu().numpy(), want, what=f"decode {geom}")


@pytest.mark.parametrize("dtype", [torch.bfloat16])
def test_decode_bf16(cuda, orc, dtype):
    q, kq, vq = make_case(2, 16, 8, 900, 256, 256, dtype=dtype, cuda=cuda, seed=5)
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 256 ** -0.5, None)
    want = oracle(orc, q, kq, vq, 256 ** -0.5, causal=False)
    assert_close_out(got.float().cpu().numpy(), want, got.dtype, what="bf16 decode")
    # fp32 output avoids the bf16 output rounding: then the 2e-3 / 1e-3 bound holds
    view, N = pkg.kernels.contiguous_view(kq, vq)
    out = pkg.kernels.attention(view, q.to(cuda), 256 ** -0.5,
                                torch.full((2,), N, dtype=torch.int32, device=cuda), N,
                                out_dtype=torch.float32)
    assert_close(out.cpu().numpy(), want, what="bf16 decode fp32 out")


def test_decode_small_l_causal(cuda, orc):
    """L = 4 query tokens (speculative-style) with the causal string mask."""
    q, kq, vq = make_case(2, 8, 2, 400, 128, 128, L=4, cuda=cuda, seed=9)
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 0.1, "causal")
    want = oracle(orc, q, kq, vq, 0.1, causal=True)
    assert_close(got.float().cpu().numpy(), want, what="causal L=4")


def test_decode_bool_and_additive_masks(cuda, orc):
    B, Hq, Hkv, N, D = 2, 8, 4, 300, 128
    q, kq, vq = make_case(B, Hq, Hkv, N, D, D, cuda=cuda, seed=13)
    g = torch.Generator().manual_seed(1)
    keep = torch.rand(B, 1, 1, N, generator=g) > 0.3
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, D ** -0.5, keep.to(cuda))
    want = oracle(orc, q, kq, vq, D ** -0.5, causal=False, mask=keep.numpy(), mask_kind=1)
    assert_close(got.float().cpu().numpy(), want, what="bool mask")
    add = torch.randn(B, 1, 1, N, generator=g).half()
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, D ** -0.5, add.to(cuda))
    want = oracle(orc, q, kq, vq, D ** -0.5, causal=False, mask=add.float().numpy(), mask_kind=2)
    assert_close(got.float().cpu().numpy(), want, what="additive mask")


def test_decode_fully_masked_row_is_uniform(cuda, orc):
    """A boolean mask that hides every key gives the uniform average (reference semantics:
    where(mask, s, finfo.min) then softmax)."""
    q, kq, vq = make_case(1, 4, 2, 50, 64, 64, cuda=cuda, seed=2)
    keep = torch.zeros(1, 1, 1, 50, dtype=torch.bool)
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 0.125, keep.to(cuda))
    want = oracle(orc, q, kq, vq, 0.125, causal=False, mask=keep.numpy(), mask_kind=1)
    assert_close(got.float().cpu().numpy(), want, what="fully masked")


@pytest.mark.parametrize("geom", [(16, 8, 256), (32, 8, 128), (8, 8, 64), (16, 16, 192)],
                         ids=["gemma256", "llama128_gqa4", "mha64", "mla192"])
@pytest.mark.parametrize("window", [0, 64, 1024])
def test_decode_left_padding_and_window(cuda, orc, window, geom):
    """Structured mask from BatchQuantizedKVCache.make_mask: left padding + sliding window,
    for GQA, MHA and MLA geometries."""
    Hq, Hkv, D = geom
    B, N = 3, 1500
    if D == 192:
        q, kq, vq = make_case(B, Hq, Hkv, N, 192, 128, cuda=cuda, seed=window + 7)
        lp = torch.tensor([0, 37, 700], dtype=torch.int64)
        mask = pkg.CausalMask(1, N - 1, window if window else None, lp)
        got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 192 ** -0.5, mask)
        want = oracle(orc, q, kq, vq, 192 ** -0.5, causal=True, window=window, kv_start=lp.numpy())
        assert_close(got.float().cpu().numpy(), want, what=f"mla left pad window={window}")
        return
    q, kq, vq = make_case(B, Hq, Hkv, N, D, D, cuda=cuda, seed=window + 1)
    lp = torch.tensor([0, 37, 700], dtype=torch.int64)
    mask = pkg.CausalMask(1, N - 1, window if window else None, lp)
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, D ** -0.5, mask)
    want = oracle(orc, q, kq, vq, D ** -0.5, causal=True, window=window, kv_start=lp.numpy())
    assert_close(got.float().cpu().numpy(), want, what=f"left pad window={window}")
    # the dense form of the same mask gives the same answer
    dense = mask.to_dense(cuda)
    got2 = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, D ** -0.5, dense)
    assert_close(got2.float().cpu().numpy(), want, what="dense form")


@pytest.mark.parametrize("n,window", [(1027, 100), (1026, 99), (2047, 113), (700, 129), (4000, 1000)])
def test_decode_window_stage_alignment(cuda, orc, n, window):
    """The first visible key is rounded down to a pipeline stage boundary (32 or 64 tokens),
    which can add up to a stage of keys to a window's span: spans that cross a chunk
    boundary only after that rounding still attend every key of the window."""
    q, kq, vq = make_case(1, 4, 1, n, 128, 128, cuda=cuda, seed=n + window)
    lp = torch.zeros(1, dtype=torch.int64)
    mask = pkg.CausalMask(1, n - 1, window, lp)
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 128 ** -0.5, mask)
    want = oracle(orc, q, kq, vq, 128 ** -0.5, causal=True, window=window, kv_start=lp.numpy())
    assert_close(got.float().cpu().numpy(), want, what=f"n={n} window={window}")


def test_batch_split_consistency(cuda):
    """B=1 and B=2 calls agree (tests/mlx/test_fused_attention_gpu.py:289-310, atol 1e-3)."""
    q, kq, vq = make_case(2, 16, 8, 640, 128, 128, cuda=cuda, seed=4)
    both = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 0.09, None)
    for b in range(2):
        one = pkg.quantized_scaled_dot_product_attention(
            q[b:b + 1].to(cuda), tuple(t[b:b + 1] for t in kq), tuple(t[b:b + 1] for t in vq), 0.09, None)
        assert torch.allclose(one.float(), both[b:b + 1].float(), atol=1e-3, rtol=0)


def test_paged_matches_contiguous(cuda, orc):
    """The same tokens stored in scattered 256-token blocks give the same output."""
    A, Hq, Hkv, D, bt = 3, 32, 8, 128, 256
    lens = [1000, 2600, 77]
    g = torch.Generator().manual_seed(7)
    nb = 40
    pool = pkg.PagedQ4Pool(Hkv, D, D, nb, bt, torch.float16, cuda)
    perm = torch.randperm(nb, generator=g)
    maxb = max(-(-n // bt) for n in lens)
    table = torch.full((A, maxb), -1, dtype=torch.int32)
    used = 0
    for a, n in enumerate(lens):
        nbk = -(-n // bt)
        table[a, :nbk] = perm[used:used + nbk]
        used += nbk
    tab = table.to(cuda)
    ks, vs = [], []
    for a, n in enumerate(lens):
        k = torch.randn(1, Hkv, n, D, generator=g).half()
        v = torch.randn(1, Hkv, n, D, generator=g).half()
        ks.append(k)
        vs.append(v)
        pkg.kernels.append(pool.view(tab[a:a + 1].contiguous()), k.to(cuda), v.to(cuda),
                           torch.zeros(1, dtype=torch.int32, device=cuda))
    q = torch.randn(A, Hq, 1, D, generator=g).half()
    kv_len = torch.tensor(lens, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(pool.view(tab), q.to(cuda), D ** -0.5, kv_len, max(lens))
    # oracle over the paged layout
    pk = tuple(_bits(t) for t in pool.k)
    pv = tuple(_bits(t) for t in pool.v)
    want = orc.attention(q.float().numpy(), pk, pv, D ** -0.5, n_kv_heads=Hkv, layout=1,
                         block_table=table.numpy(), kv_len=np.array(lens), causal=False)
    assert_close(got.float().cpu().numpy(), want, what="paged")
    # and each agent alone through the contiguous path
    for a, n in enumerate(lens):
        kq, vq = pkg.quantize(ks[a].to(cuda)), pkg.quantize(vs[a].to(cuda))
        one = pkg.quantized_scaled_dot_product_attention(q[a:a + 1].to(cuda), kq, vq, D ** -0.5, None)
        assert torch.allclose(one.float(), got[a:a + 1].float(), atol=2e-3, rtol=1e-3)


def test_paged_bad_block_is_flagged_not_read(cuda):
    pool = pkg.PagedQ4Pool(2, 128, 128, 4, 256, torch.float16, cuda)
    table = torch.tensor([[1, 12345]], dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    q = torch.randn(1, 4, 1, 128, dtype=torch.float16, device=cuda)
    out = pkg.kernels.attention(pool.view(table), q, 0.1, torch.tensor([400], dtype=torch.int32, device=cuda),
                                400, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
    assert torch.isfinite(out.float()).all()


def test_unsupported_dims_raise(cuda):
    q, kq, vq = make_case(1, 2, 1, 20, 320, 320, cuda=cuda)
    with pytest.raises(pkg.Q4KernelError):
        pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 0.1, None)


def test_cluster_merge_needs_no_workspace(cuda, merge_mode):
    """Split chunks that fit one cluster merge there (no workspace); with cluster merging
    turned off the same call needs a workspace for its partials."""
    L_ = pkg._lib.load()
    q, kq, vq = make_case(2, 32, 8, 2048, 128, 128, cuda=cuda, seed=1)
    view, _ = pkg.kernels.contiguous_view(kq, vq)
    a = pkg._lib.AttnArgs()
    a.batch, a.n_q_heads, a.q_len, a.max_kv_len = 2, 32, 1, 2048
    a.scale = 128 ** -0.5
    ws = L_.am_q4_attention_workspace_bytes(ctypes.byref(view.desc), ctypes.byref(a))
    if merge_mode == "cluster":
        assert ws == 0
    else:
        assert ws > 0


def test_decode_full_chunks_accuracy(cuda, orc, merge_mode):
    """Enough (sequence, KV head) pairs to fill the device, so every CTA streams a whole
    8192-token chunk: the longest fp32 accumulation of the kernel (the V accumulators hold
    whole code bytes and are separated by a subtraction at the end) stays within tolerance."""
    B, Hq, Hkv, N, D = 64, 32, 8, 8192, 128
    g = torch.Generator(device=cuda).manual_seed(11)
    k = torch.randn(B, Hkv, N, D, generator=g, device=cuda, dtype=torch.float16)
    v = torch.randn(B, Hkv, N, D, generator=g, device=cuda, dtype=torch.float16)
    q = torch.randn(B, Hq, 1, D, generator=g, device=cuda, dtype=torch.float16)
    kq, vq = pkg.quantize(k), pkg.quantize(v)
    del k, v
    got = pkg.quantized_scaled_dot_product_attention(q, kq, vq, D ** -0.5, None)
    want = oracle(orc, q.cpu(), tuple(t.cpu() for t in kq), tuple(t.cpu() for t in vq), D ** -0.5,
                  causal=False)
    g32 = got.float().cpu().numpy()
    print(f"8192-token chunks ({merge_mode}): max abs err {np.abs(g32 - want).max():.2e}")
    assert_close(g32, want, what="8192-token chunks")


def test_pool_beyond_tensor_map_rows_is_refused(cuda):
    """A pool descriptor claiming more than 2^31 code rows is refused before any launch (the
    TMA coordinates of a row are 32-bit); nothing is read or written."""
    pool = pkg.PagedQ4Pool(2, 128, 128, 4, 256, torch.float16, cuda)
    table = torch.tensor([[0, 1]], dtype=torch.int32, device=cuda)
    view = pool.view(table)
    view.desc.capacity = (1 << 31) // (2 * 256) + 1  # num_blocks x heads x tokens > 2^31
    q = torch.randn(1, 4, 1, 128, dtype=torch.float16, device=cuda)
    out = torch.full((1, 4, 1, 128), 7.0, dtype=torch.float16, device=cuda)
    with pytest.raises(pkg.Q4KernelError, match="code rows"):
        pkg.kernels.attention(view, q, 0.1, torch.tensor([300], dtype=torch.int32, device=cuda), 300,
                              out=out, mode="decode")
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
