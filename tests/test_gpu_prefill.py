"""GPU parity of the tcgen05 chunked-prefill kernel against the CPU oracle.

Tolerance: |gpu - oracle| <= 2e-3 + 1e-3 * |oracle| (fp32 output), fp32 accumulation in
TMEM.  The chunk's own K/V are quantized into the cache before attention, as in the
reference's chunked prefill (quantize-on-append precedes the attention call).
"""

import numpy as np
import pytest
import torch

from conftest import assert_close, assert_close_out, pkg
from test_gpu_decode import _bits, make_case, oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qdtype", [torch.float16, torch.bfloat16])
def test_prefill_llama_gqa(cuda, orc, qdtype):
    """Llama-3.1-8B head geometry (32/8, D128), 512-token chunk over a cached prefix."""
    B, Hq, Hkv, D, L, P = 2, 32, 8, 128, 512, 600
    N = P + L
    q, kq, vq = make_case(B, Hq, Hkv, N, D, D, L=L, dtype=qdtype, cuda=cuda, seed=41)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), D ** -0.5, kv_len, N, causal=True,
                                out_dtype=torch.float32, mode="prefill")
    want = oracle(orc, q, kq, vq, D ** -0.5, causal=True)
    assert_close(got.cpu().numpy(), want, what=f"prefill {qdtype}")


def test_prefill_through_dropin_op(cuda, orc):
    """The drop-in op routes L=64 with the causal string to the prefill kernel; its fp16
    output is held to the attention bound plus fp16's own rounding, and the same call with
    fp32 output to the attention bound alone."""
    q, kq, vq = make_case(1, 8, 8, 300, 128, 128, L=64, cuda=cuda, seed=3)
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, 0.08, "causal")
    want = oracle(orc, q, kq, vq, 0.08, causal=True)
    assert got.dtype == torch.float16
    assert_close_out(got.float().cpu().numpy(), want, got.dtype, what="drop-in prefill")
    view, N = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((1,), N, dtype=torch.int32, device=cuda)
    got32 = pkg.kernels.attention(view, q.to(cuda), 0.08, kv_len, N, causal=True,
                                  out_dtype=torch.float32)
    assert_close(got32.cpu().numpy(), want, what="drop-in prefill, fp32 out")


def test_prefill_d64_mha_window_leftpad(cuda, orc):
    B, H, D, L, N = 3, 4, 64, 200, 700
    q, kq, vq = make_case(B, H, H, N, D, D, L=L, cuda=cuda, seed=8)
    lp = torch.tensor([0, 5, 301])
    view, _ = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), 0.125, kv_len, N, causal=True, window=128,
                                kv_start=lp.to(cuda), out_dtype=torch.float32, mode="prefill")
    want = oracle(orc, q, kq, vq, 0.125, causal=True, window=128, kv_start=lp.numpy())
    assert_close(got.cpu().numpy(), want, what="prefill window+leftpad")


def test_prefill_dense_masks(cuda, orc):
    B, H, D, L, N = 1, 4, 128, 130, 260
    q, kq, vq = make_case(B, H, 2, N, D, D, L=L, cuda=cuda, seed=10)
    g = torch.Generator().manual_seed(0)
    keep = torch.rand(B, 1, L, N, generator=g) > 0.2
    view, _ = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), 0.1, kv_len, N, mask=keep.to(cuda),
                                out_dtype=torch.float32, mode="prefill")
    want = oracle(orc, q, kq, vq, 0.1, causal=False, mask=keep.numpy(), mask_kind=1)
    assert_close(got.cpu().numpy(), want, what="prefill bool mask")


def test_prefill_matches_decode_kernel(cuda):
    """Both kernels agree on a 16-query block (the dispatch boundary)."""
    q, kq, vq = make_case(2, 4, 1, 900, 128, 128, L=16, cuda=cuda, seed=12)
    view, N = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((2,), N, dtype=torch.int32, device=cuda)
    a = pkg.kernels.attention(view, q.to(cuda), 0.09, kv_len, N, causal=True,
                              out_dtype=torch.float32, mode="prefill")
    b = pkg.kernels.attention(view, q.to(cuda), 0.09, kv_len, N, causal=True,
                              out_dtype=torch.float32, mode="decode")
    assert torch.allclose(a, b, atol=2e-3, rtol=1e-3), (a - b).abs().max()


@pytest.mark.parametrize("geom", [(2, 32, 8, 128, 128, 700, 300), (2, 16, 8, 256, 256, 420, 200),
                                  (2, 16, 16, 192, 128, 330, 190)],
                         ids=["llama_d128", "gemma_d256", "mla_k192_v128"])
def test_chunked_prefill_paged(cuda, orc, geom):
    """Config-4 flow at reduced size on the paged pool: append the chunk's K/V into
    256-token blocks, then attend the chunk over prefix + chunk.  The Gemma-3 and MLA
    geometries take the kernel that dequantizes its tiles from the pool blocks itself
    (tiles that straddle two blocks, bf16 scales)."""
    A, Hq, Hkv, Dk, Dv, P, L = geom
    bt = 256
    spec = pkg.ModelCacheSpec(n_layers=1, n_kv_heads=Hkv, head_dim=Dk, block_tokens=bt,
                              layer_types=["global"], v_head_dim=Dv)
    alloc = pkg.shuffled_allocator(spec, 32, seed=1)
    pool = pkg.PagedQ4Pool.for_spec(spec, 32, torch.bfloat16, cuda)
    layer = pkg.PagedLayerCache(pool, alloc, 0, ["a0", "a1"][:A], P + L)
    g = torch.Generator().manual_seed(2)
    kp = torch.randn(A, Hkv, P, Dk, generator=g).bfloat16()
    vp = torch.randn(A, Hkv, P, Dv, generator=g).bfloat16()
    layer.append(kp.to(cuda), vp.to(cuda))
    kc = torch.randn(A, Hkv, L, Dk, generator=g).bfloat16()
    vc = torch.randn(A, Hkv, L, Dv, generator=g).bfloat16()
    layer.append(kc.to(cuda), vc.to(cuda))
    q = torch.randn(A, Hq, L, Dk, generator=g).bfloat16()
    got = layer.attention(q.to(cuda), Dk ** -0.5, mode="prefill")
    table = layer._table_host.numpy()
    want = orc.attention(q.float().numpy(), tuple(_bits(t) for t in pool.k),
                         tuple(_bits(t) for t in pool.v), Dk ** -0.5, sdtype=1, n_kv_heads=Hkv,
                         layout=1, block_table=table, kv_len=np.array(layer.lengths), causal=True)
    assert got.dtype == torch.bfloat16
    assert_close_out(got.float().cpu().numpy(), want, got.dtype, what="paged chunked prefill")
    out32 = torch.empty(A, Hq, L, Dv, dtype=torch.float32, device=cuda)
    layer.attention(q.to(cuda), Dk ** -0.5, out=out32, mode="prefill")
    assert_close(out32.cpu().numpy(), want, what="paged chunked prefill, fp32 out")


@pytest.mark.parametrize("geom", [(2, 16, 8, 256, 256, 100), (1, 16, 16, 192, 128, 80),
                                  (2, 8, 4, 128, 64, 90)],
                         ids=["gemma_d256", "mla_k192_v128", "k128_v64"])
@pytest.mark.parametrize("window", [0, 96])
def test_prefill_gemma_mla_geometries(cuda, orc, geom, window):
    """Query blocks on the Gemma-3 (D256, 64-key tiles), MLA (K192 / V128) and asymmetric
    geometries: causal, sliding window, left padding."""
    B, Hq, Hkv, dk, dv, L = geom
    P = 150
    N = P + L
    q, kq, vq = make_case(B, Hq, Hkv, N, dk, dv, L=L, cuda=cuda, seed=dk + L + window)
    lp = torch.tensor([0, 7][:B])
    view, _ = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), dk ** -0.5, kv_len, N, causal=True, window=window,
                                kv_start=lp.to(cuda), out_dtype=torch.float32, mode="prefill")
    want = oracle(orc, q, kq, vq, dk ** -0.5, causal=True, window=window, kv_start=lp.numpy())
    assert_close(got.cpu().numpy(), want, what=f"prefill {geom} window={window}")


def test_prefill_d256_dense_mask(cuda, orc):
    """Non-causal query block with a boolean mask on a D256 cache."""
    B, Hq, Hkv, D, L, N = 1, 8, 4, 256, 70, 200
    q, kq, vq = make_case(B, Hq, Hkv, N, D, D, L=L, cuda=cuda, seed=77)
    g = torch.Generator().manual_seed(1)
    keep = torch.rand(B, 1, L, N, generator=g) > 0.3
    view, _ = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), 0.06, kv_len, N, mask=keep.to(cuda),
                                out_dtype=torch.float32, mode="prefill")
    want = oracle(orc, q, kq, vq, 0.06, causal=False, mask=keep.numpy(), mask_kind=1)
    assert_close(got.cpu().numpy(), want, what="prefill d256 dense mask")


@pytest.mark.parametrize("geom", [(2, 16, 8, 256, 256), (1, 16, 16, 192, 128)], ids=["gemma", "mla"])
def test_prefill_reference_short_blocks(cuda, orc, geom):
    """The reference's own tests drive Gemma-like and DeepSeek-like query blocks of L = 2
    (tests/mlx/test_fused_attention_gpu.py:648-674): the drop-in op takes them through the
    decode kernel; forcing the prefill kernel gives the same answer."""
    B, Hq, Hkv, dk, dv = geom
    q, kq, vq = make_case(B, Hq, Hkv, 300, dk, dv, L=2, cuda=cuda, seed=5)
    want = oracle(orc, q, kq, vq, dk ** -0.5, causal=True)
    got = pkg.quantized_scaled_dot_product_attention(q.to(cuda), kq, vq, dk ** -0.5, "causal")
    assert_close_out(got.float().cpu().numpy(), want, got.dtype, what="L=2 drop-in")
    view, N = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got2 = pkg.kernels.attention(view, q.to(cuda), dk ** -0.5, kv_len, N, causal=True,
                                 out_dtype=torch.float32, mode="prefill")
    assert_close(got2.cpu().numpy(), want, what="L=2 prefill kernel")


def test_prefill_ragged_kv_len(cuda, orc):
    """Sequences shorter than the max_kv_len the workspace was sized for: the rows past a
    sequence's end in its workspace plane are zeros and every output stays finite."""
    B, Hq, Hkv, D, L, N = 2, 8, 2, 128, 64, 500
    q, kq, vq = make_case(B, Hq, Hkv, N, D, D, L=L, cuda=cuda, seed=31)
    view, _ = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.tensor([N, 300], dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), 0.09, kv_len, N, causal=True,
                                out_dtype=torch.float32, mode="prefill")
    assert torch.isfinite(got).all()
    want = oracle(orc, q, kq, vq, 0.09, causal=True, kv_len=np.array([N, 300]))
    assert_close(got.cpu().numpy(), want, what="ragged kv_len")


@pytest.mark.parametrize("trend", ["rising", "falling"])
@pytest.mark.parametrize("dims", [(128, 128), (192, 128), (256, 256)], ids=["d128", "k192_v128", "d256"])
def test_prefill_scores_that_jump_between_tiles(cuda, orc, trend, dims):
    """Scores that jump by ~40 (log2 units) from one 128-key tile to the next, rising or
    falling along the keys: the one-pass softmax must detect a running max that has fallen
    behind (a tile sum beyond the fp16 range of P) and redo the tile after a max pass and
    rescale; falling scores keep the first tiles' max and give tiny P.  Every key is a
    constant vector a_t (a multiple of 1/8 below 32), which Q4 and the fp16 operands both
    hold exactly, so large scores carry no operand rounding; the queries are |N(0,1)|, so
    q . k grows with a_t."""
    B, Hq, Hkv, L, P = 1, 8, 2, 256, 1024
    dk, dv = dims
    N = P + L
    t = torch.arange(N)
    a = 2.5 * (t // 128).float() + ((t * 5) % 8).float() / 8.0
    if trend == "falling":
        a = a.flip(0)
    g = torch.Generator().manual_seed(57)
    k = a[None, None, :, None].expand(B, Hkv, N, dk).half().contiguous()
    v = torch.randn(B, Hkv, N, dv, generator=g).half()
    q = torch.randn(B, Hq, L, dk, generator=g).abs().half()
    kq, vq = pkg.quantize(k.to(cuda)), pkg.quantize(v.to(cuda))
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), dk ** -0.5, kv_len, N, causal=True,
                                out_dtype=torch.float32, mode="prefill")
    want = oracle(orc, q, kq, vq, dk ** -0.5, causal=True)
    assert_close(got.cpu().numpy(), want, what=f"prefill {trend} scores {dims}")


@pytest.mark.parametrize("geom", [(4, 4, 192, 128), (8, 4, 256, 256)], ids=["k192_v128", "d256"])
def test_prefill_values_beyond_fp16_saturate(cuda, orc, geom):
    """A bf16 cache can hold groups whose dequantized values leave fp16's range.  Every
    prefill path saturates them at +-65504 (the attention kernels' fp16 operands): the K
    plane in the stage kernel, and for these head dims the V tiles dequantized inside the
    attention kernel, whose f16x2 conversion hands such groups to an fp32 path.  Keys a
    query cannot see therefore still contribute exactly 0 (no 0 * inf), and the outputs
    match an fp64 attention over the saturated values."""
    Hq, Hkv, dk, dv = geom
    B, N, L = 1, 300, 100
    g = torch.Generator().manual_seed(17)
    k = torch.randn(B, Hkv, N, dk, generator=g)
    v = torch.randn(B, Hkv, N, dv, generator=g)
    # keys 250..269 (visible to queries at positions >= 250 only): the first 64-element V
    # group spans 5e4 .. 9e4, so codes above ~6 dequantize beyond 65504
    v[:, :, 250:270, :64] = 5.0e4 + 4.0e4 * torch.rand(B, Hkv, 20, 64, generator=g)
    v[:, :, 250:270, 0] = 5.0e4
    v[:, :, 250:270, 1] = 9.0e4
    kq = pkg.quantize(k.bfloat16().to(cuda))
    vq = pkg.quantize(v.bfloat16().to(cuda))
    q = torch.randn(B, Hq, L, dk, generator=g).bfloat16()
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), n, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q.to(cuda), dk ** -0.5, kv_len, n, causal=True,
                                out_dtype=torch.float32, mode="prefill")
    assert torch.isfinite(got).all()
    sat = lambda x: np.clip(x.astype(np.float64), -65504.0, 65504.0)
    kd = sat(orc.dequantize(*(_bits(t) for t in kq), dtype=1))  # [B, Hkv, N, dk]
    vd = sat(orc.dequantize(*(_bits(t) for t in vq), dtype=1))
    qf = q.float().numpy().astype(np.float64)
    n_rep = Hq // Hkv
    want = np.zeros((B, Hq, L, dv))
    for hq in range(Hq):
        s = qf[0, hq] @ kd[0, hq // n_rep].T * dk ** -0.5  # [L, N]
        pos = N - L + np.arange(L)
        s[np.arange(N)[None, :] > pos[:, None]] = -np.inf
        p = np.exp(s - s.max(axis=1, keepdims=True))
        want[0, hq] = (p / p.sum(axis=1, keepdims=True)) @ vd[0, hq // n_rep]
    assert np.abs(want).max() > 1.0e4  # the saturated keys carry weight for later queries
    assert_close(got.cpu().numpy(), want, what=f"prefill {geom}, V beyond the fp16 range")


@pytest.mark.parametrize("geom", [(2, 32, 8, 128, 128, 1112, 512, 0, 600),
                                  (2, 16, 16, 192, 128, 520, 190, 0, 333),
                                  (2, 16, 8, 256, 256, 620, 200, 128, 517)],
                         ids=["llama_d128", "mla_k192_v128", "gemma_d256_window"])
def test_prefill_stage_then_attend_matches_prefill(cuda, geom):
    """am_q4_prefill_stage over two key ranges (the later range first, split inside a stage
    CTA's rows) then am_q4_prefill_attend give exactly am_q4_prefill's outputs, over a
    workspace filled with all-ones bytes (NaN as fp16) beforehand, so a row that no stage
    call wrote would show."""
    B, Hq, Hkv, Dk, Dv, N, L, window, split = geom
    q, kq, vq = make_case(B, Hq, Hkv, N, Dk, Dv, L=L, cuda=cuda, seed=17)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    qd = q.to(cuda)
    kw = dict(causal=True, window=window, out_dtype=torch.float32)
    want = pkg.kernels.attention(view, qd, Dk ** -0.5, kv_len, N, mode="prefill", **kw)
    nbytes = pkg.kernels.prefill_workspace_bytes(view, B, Hq, L, N, window=window)
    ws = torch.full((nbytes,), 255, dtype=torch.uint8, device=cuda)
    for keys in ((split, 2 ** 31 - 1), (0, split)):
        pkg.kernels.attention(view, qd, Dk ** -0.5, kv_len, N, mode="prefill_stage",
                              workspace=ws, stage_keys=keys, **kw)
    got = pkg.kernels.attention(view, qd, Dk ** -0.5, kv_len, N, mode="prefill_attend",
                                workspace=ws, **kw)
    torch.cuda.synchronize(cuda)
    assert torch.equal(got, want), (got - want).abs().max()


@pytest.mark.parametrize("geom", [(2, 32, 8, 128, 128, 700, 300, 0),
                                  (2, 16, 8, 256, 256, 420, 200, 96),
                                  (2, 16, 16, 192, 128, 330, 190, 0)],
                         ids=["llama_d128", "gemma_d256_window", "mla_k192_v128"])
def test_paged_prefill_stage_before_append_then_attend(cuda, geom):
    """The serving order of the split prefill on the paged pool (bf16 scales, shuffled
    256-token blocks): the cached prefix is staged BEFORE the chunk's K/V are appended (as
    the bench's side stream does while the previous layer runs), then the chunk is appended,
    its rows staged and attended; the outputs equal am_q4_prefill's after the append, bit
    for bit, over a workspace filled with NaN bytes beforehand."""
    A, Hq, Hkv, Dk, Dv, P, L, window = geom
    bt = 256
    spec = pkg.ModelCacheSpec(n_layers=1, n_kv_heads=Hkv, head_dim=Dk, block_tokens=bt,
                              layer_types=["global"], v_head_dim=Dv)
    alloc = pkg.shuffled_allocator(spec, 32, seed=3)
    pool = pkg.PagedQ4Pool.for_spec(spec, 32, torch.bfloat16, cuda)
    layer = pkg.PagedLayerCache(pool, alloc, 0, ["a0", "a1"][:A], P + L)
    g = torch.Generator().manual_seed(5)
    layer.append(torch.randn(A, Hkv, P, Dk, generator=g).bfloat16().to(cuda),
                 torch.randn(A, Hkv, P, Dv, generator=g).bfloat16().to(cuda))
    kc = torch.randn(A, Hkv, L, Dk, generator=g).bfloat16().to(cuda)
    vc = torch.randn(A, Hkv, L, Dv, generator=g).bfloat16().to(cuda)
    q = torch.randn(A, Hq, L, Dk, generator=g).bfloat16().to(cuda)
    N = P + L
    for r in range(A):
        layer.reserve(r, N)
    kv_len = torch.full((A,), N, dtype=torch.int32, device=cuda)
    out = torch.empty(A, Hq, L, Dv, dtype=torch.float32, device=cuda)
    kw = dict(causal=True, window=window, out=out)
    nbytes = pkg.kernels.prefill_workspace_bytes(layer.view(), A, Hq, L, N, window=window)
    ws = torch.full((nbytes,), 255, dtype=torch.uint8, device=cuda)
    pkg.kernels.attention(layer.view(), q, Dk ** -0.5, kv_len, N, mode="prefill_stage",
                          workspace=ws, stage_keys=(0, P), **kw)
    layer.append(kc, vc)  # writes positions P .. N - 1 only
    pkg.kernels.attention(layer.view(), q, Dk ** -0.5, kv_len, N, mode="prefill_stage",
                          workspace=ws, stage_keys=(P, 2 ** 31 - 1), **kw)
    pkg.kernels.attention(layer.view(), q, Dk ** -0.5, kv_len, N, mode="prefill_attend",
                          workspace=ws, **kw)
    got = out.clone()
    want = pkg.kernels.attention(layer.view(), q, Dk ** -0.5, kv_len, N, mode="prefill",
                                 causal=True, window=window, out_dtype=torch.float32)
    torch.cuda.synchronize(cuda)
    assert torch.equal(got, want), (got - want).abs().max()
