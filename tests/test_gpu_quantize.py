"""GPU parity of quantize / dequantize / quantize-on-append against the CPU oracle.

Integer outputs (codes) and the fp16/bf16 scales and biases must be bit-identical to the
oracle's restatement of mlx's affine quantizer.
"""

import numpy as np
import pytest
import torch

from conftest import pkg

pytestmark = pytest.mark.gpu

F16, BF16 = 0, 1


def _bits(t: torch.Tensor) -> np.ndarray:
    a = t.detach().cpu()
    if a.dtype == torch.int32:
        return a.numpy().view(np.uint32)
    return a.view(torch.int16).numpy().view(np.uint16)


def _rand(shape, dtype, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def _oracle_q(x: torch.Tensor, orc):
    dt = BF16 if x.dtype == torch.bfloat16 else F16
    return orc.quantize(x.view(torch.int16).numpy().view(np.uint16), dt)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 64), (7, 128), (3, 5, 192), (2, 8, 33, 256), (4096, 128)])
def test_quantize_bit_exact(cuda, orc, dtype, shape):
    x = _rand(shape, dtype, seed=hash(shape) % 1000)
    got = pkg.quantize(x.to(cuda))
    want = _oracle_q(x, orc)
    assert got[0].shape == want[0].shape and got[1].dtype == dtype
    for g, w, name in zip(got, want, ("codes", "scales", "biases")):
        np.testing.assert_array_equal(_bits(g), w.view(np.uint32 if name == "codes" else np.uint16),
                                      err_msg=name)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quantize_edge_groups(cuda, orc, dtype):
    """Degenerate groups: zeros, constants, single outlier, negative-dominant, tiny values,
    large magnitudes, exact ties."""
    rows = []
    rows.append(torch.zeros(64))
    rows.append(torch.full((64,), 3.0))
    rows.append(torch.full((64,), -2.5))
    r = torch.zeros(64); r[17] = 100.0; rows.append(r)
    r = torch.linspace(-7, 1, 64); rows.append(r)
    r = torch.linspace(-1, 7, 64); rows.append(r)
    rows.append(torch.full((64,), 1e-6))
    r = torch.linspace(-3e-5, 3e-5, 64); rows.append(r)
    r = torch.linspace(-60000, 60000, 64) if dtype == torch.float16 else torch.linspace(-1e30, 1e30, 64)
    rows.append(r)
    rows.append(torch.arange(64, dtype=torch.float32) % 16)  # exact codes
    rows.append((torch.arange(64, dtype=torch.float32) % 16) * 0.5 + 0.25)
    x = torch.stack(rows).to(dtype)
    got = pkg.quantize(x.to(cuda))
    want = _oracle_q(x, orc)
    for g, w, name in zip(got, want, ("codes", "scales", "biases")):
        np.testing.assert_array_equal(_bits(g), w.view(np.uint32 if name == "codes" else np.uint16),
                                      err_msg=name)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dequantize_matches_oracle(cuda, orc, dtype):
    x = _rand((300, 128), dtype, seed=3)
    q = pkg.quantize(x.to(cuda))
    got = pkg.dequantize(*q, dtype=torch.float32).cpu().numpy()
    dt = BF16 if dtype == torch.bfloat16 else F16
    want = orc.dequantize(*[_bits(t) for t in q], dtype=dt)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-6 * np.abs(want).max())
    # round trip error bounded by the group's step (plus the clamp of mlx's zero-exact rule)
    err = np.abs(got - x.float().numpy())
    assert err.max() < 0.5


def test_quantize_rejects_bad_dim(cuda):
    with pytest.raises(ValueError):
        pkg.quantize(torch.zeros(4, 96, dtype=torch.float16, device=cuda))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("dims", [(128, 128), (192, 128), (256, 256), (64, 64)])
def test_append_contiguous(cuda, orc, dtype, dims):
    dk, dv = dims
    B, H, L, cap = 3, 4, 37, 256
    k = _rand((B, H, L, dk), dtype, 11)
    v = _rand((B, H, L, dv), dtype, 12)
    keys = tuple(t.to(cuda) for t in (torch.zeros(B, H, cap, dk // 8, dtype=torch.int32),
                                      torch.zeros(B, H, cap, dk // 64, dtype=dtype),
                                      torch.zeros(B, H, cap, dk // 64, dtype=dtype)))
    vals = tuple(t.to(cuda) for t in (torch.zeros(B, H, cap, dv // 8, dtype=torch.int32),
                                      torch.zeros(B, H, cap, dv // 64, dtype=dtype),
                                      torch.zeros(B, H, cap, dv // 64, dtype=dtype)))
    view, _ = pkg.kernels.contiguous_view(keys, vals)
    pos = torch.tensor([0, 100, 219], dtype=torch.int32, device=cuda)
    pkg.kernels.append(view, k.to(cuda), v.to(cuda), pos)
    wk, wv = _oracle_q(k, orc), _oracle_q(v, orc)
    for b, p in enumerate([0, 100, 219]):
        for got, want in ((keys, wk), (vals, wv)):
            for g, w in zip(got, want):
                np.testing.assert_array_equal(_bits(g[b, :, p:p + L]), w[b].view(_bits(g).dtype))
        # untouched rows stay zero
        assert _bits(keys[0][b, :, p + L:]).sum() == 0 if p + L < cap else True


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_append_paged_scatter(cuda, orc, dtype):
    nb, H, bt, D = 40, 2, 256, 128
    pool = pkg.PagedQ4Pool(H, D, D, nb, bt, dtype, cuda)
    table = torch.tensor([[5, 17, 3, -1], [22, 0, 39, 8]], dtype=torch.int32)
    A, L = 2, 300
    k = _rand((A, H, L, D), dtype, 21)
    v = _rand((A, H, L, D), dtype, 22)
    pos = torch.tensor([10, 200], dtype=torch.int32)
    pkg.kernels.append(pool.view(table.to(cuda)), k.to(cuda), v.to(cuda), pos.to(cuda))
    wk, wv = _oracle_q(k, orc), _oracle_q(v, orc)
    for a in range(A):
        for l in range(L):
            t = int(pos[a]) + l
            blk = int(table[a, t // bt])
            for got, want in ((pool.k, wk), (pool.v, wv)):
                for g, w in zip(got, want):
                    np.testing.assert_array_equal(_bits(g[blk, :, t % bt]), w[a, :, l].view(_bits(g).dtype))


def test_append_flags_bad_block(cuda):
    pool = pkg.PagedQ4Pool(1, 64, 64, 4, 16, torch.float16, cuda)
    table = torch.tensor([[0, 99]], dtype=torch.int32, device=cuda)  # block 99 does not exist
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    k = torch.randn(1, 1, 32, 64, dtype=torch.float16, device=cuda)
    pkg.kernels.append(pool.view(table), k, k, torch.zeros(1, dtype=torch.int32, device=cuda), status)
    assert int(status.item()) & 1  # AM_STATUS_BAD_BLOCK
    # the valid block was still written
    assert _bits(pool.k[0][0]).any()


def _edge_rows(dtype):
    """Groups at the corners of the affine rule (mlx 0.30.3 affine quantizer: in the mlx
    sources mlx/backend/cpu/quantized.cpp and the Metal kernel's affine_quantize): exact
    round-half ties of (w - bias) / scale, groups whose q0 = rint(edge / scale) is 0, constant
    groups, the dtype's largest finite values, and subnormal inputs."""
    f32 = torch.float32
    rows = []
    # ties: min -15, max 0 -> scale 1, bias -15, (w - bias) / scale = k + 0.5 exactly
    t = torch.tensor([-15.0 + (k % 15) + 0.5 for k in range(64)], dtype=f32)
    t[0], t[1] = -15.0, 0.0
    rows.append(t)
    # the same with a power-of-two step: min -7.5, max 0 -> scale 0.5, ties at j * 0.5 + 0.25
    t = torch.tensor([-7.5 + (k % 15) * 0.5 + 0.25 for k in range(64)], dtype=f32)
    t[0], t[1] = -7.5, 0.0
    rows.append(t)
    # ties on the max side (scale negative): max 15, min 0
    t = torch.tensor([(k % 15) + 0.5 for k in range(64)], dtype=f32)
    t[0], t[1] = 0.0, 15.0
    rows.append(t)
    # q0 = 0: an all-zero group, a group of negative zeros, and (bf16) values far below the
    # 1e-7 scale floor, whose edge / scale rounds to 0 so the bias is 0
    rows.append(torch.zeros(64, dtype=f32))
    rows.append(-torch.zeros(64, dtype=f32))
    if dtype == torch.bfloat16:
        rows.append(torch.linspace(-3e-8, 4e-8, 64, dtype=f32))
        rows.append(torch.full((64,), 2e-8, dtype=f32))
    # constants of both signs and sizes
    for c in (1.0, -1.0, 0.3333, -1234.5, 7.0e-5):
        rows.append(torch.full((64,), c, dtype=f32))
    # the largest finite values of the dtype (fp16 +-65504); for bf16 the largest values whose
    # range max - min stays finite in the rule's fp32 arithmetic (+-1.6e38: a group spanning
    # +-3.39e38 overflows to an infinite scale, in mlx as here, and has no defined codes).
    # fp16 groups of zeros get the fp16 subnormal scale -1.19e-7 (the 1e-7 floor, rounded).
    big = 65504.0 if dtype == torch.float16 else 1.6e38
    t = torch.linspace(-1, 1, 64, dtype=f32) * 1000.0
    t[3], t[40] = big, -big
    rows.append(t)
    t = torch.full((64,), big, dtype=f32)
    t[9] = -big
    rows.append(t)
    # a constant group divides its value by the 1e-7 scale floor: bf16 constants above
    # ~3.4e31 overflow that quotient (undefined codes, in mlx as here), so bf16 uses 1e30
    rows.append(torch.full((64,), -(big if dtype == torch.float16 else 1e30), dtype=f32))
    # subnormal inputs (fp16 subnormals below 6.1e-5; bf16 ones below 1.2e-38)
    tiny = 6.0e-8 if dtype == torch.float16 else 1.0e-39
    rows.append(torch.arange(64, dtype=f32) * tiny)
    rows.append((torch.arange(64, dtype=f32) - 32) * tiny)
    return torch.stack(rows).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quantize_pinned_edge_cases(cuda, orc, dtype):
    """Bit-exact GPU vs both CPU restatements on the rule's corner cases, and ties round to
    the even code (rint), the rounding the restatement follows."""
    x = _edge_rows(dtype)
    dt = BF16 if dtype == torch.bfloat16 else F16
    got = [_bits(t) for t in pkg.quantize(x.to(cuda))]
    want_c = _oracle_q(x, orc)
    want_np = orc.quantize_np(x.view(torch.int16).numpy().view(np.uint16), dt)
    for g, wc, wn, name in zip(got, want_c, want_np, ("codes", "scales", "biases")):
        kind = np.uint32 if name == "codes" else np.uint16
        np.testing.assert_array_equal(g, wc.view(kind), err_msg=f"{name} vs C oracle")
        np.testing.assert_array_equal(g, np.asarray(wn).view(kind), err_msg=f"{name} vs NumPy oracle")
    codes = got[0].reshape(x.shape[0], -1)
    nib = (codes[:, :, None] >> (np.arange(8, dtype=np.uint32) * 4)) & 0xF
    nib = nib.reshape(x.shape[0], 64)
    # row 0: (w + 15) = k + 0.5 -> even neighbour of k + 0.5 (k + 1 when k is odd, k when even)
    k = np.arange(64) % 15
    expect = np.where(k % 2 == 0, k, k + 1)
    np.testing.assert_array_equal(nib[0, 2:], expect[2:])
    # all-zero groups: bias 0, codes 0
    assert not nib[3].any() and not nib[4].any()
