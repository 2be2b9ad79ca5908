"""GPU parity at the benchmark configurations' own shapes (one layer each).

The other parity files run the geometries at reduced sizes; here every case has the exact
shape of a benchmark configuration, fp32 outputs and the attention tolerance
|gpu - oracle| <= 2e-3 + 1e-3 * |oracle| (fp32 accumulation):

* Gemma-3-12B decode: batch 8, 16 query / 8 KV heads, head dim 256, context 4096, one
  global layer and one sliding-window layer (window 1024);
* DeepSeek-Coder-V2-Lite MLA decode: batch 16, 16 heads, K dim 192 / V dim 128, context 8192;
* chunked prefill, Llama-3.1-8B heads (32 / 8, head dim 128): batch 2, a 512-token bf16
  chunk appended into 256-token pool blocks after a 4096-token prefix, causal attention of
  the chunk over prefix + chunk;
* 512-token chunks on the Gemma-3 (global and window-1024 layers) and MLA shapes;
* multi-agent block-pool decode, Llama-3.1-8B heads: a sample of agents whose contexts span
  the workload's range (1024 to 32768 tokens), blocks at shuffled pool offsets.

Inputs are seeded N(0,1); K/V are quantized on the GPU (bit-exact with the oracle's
quantizer, tests/test_gpu_quantize.py) and the oracle reads the same Q4 bytes.
"""

import numpy as np
import pytest
import torch

from conftest import assert_close, pkg
from test_gpu_decode import _bits

pytestmark = pytest.mark.gpu

F16, BF16 = 0, 1


def _q4_bits(q4):
    return tuple(_bits(t) for t in q4)


def _randn(shape, seed, dev, dtype=torch.float16):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(*shape, generator=g, device=dev, dtype=dtype)


@pytest.mark.usefixtures("merge_mode")
@pytest.mark.parametrize("window", [0, 1024], ids=["global", "window1024"])
def test_gemma3_decode_layer(cuda, orc, window):
    B, Hq, Hkv, D, N = 8, 16, 8, 256, 4096
    kq = pkg.quantize(_randn((B, Hkv, N, D), 1, cuda))
    vq = pkg.quantize(_randn((B, Hkv, N, D), 2, cuda))
    q = _randn((B, Hq, 1, D), 3, cuda)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q, D ** -0.5, kv_len, N, causal=True, window=window,
                                out_dtype=torch.float32, mode="decode")
    want = orc.attention(q.float().cpu().numpy(), _q4_bits(kq), _q4_bits(vq), D ** -0.5,
                         causal=True, window=window)
    assert_close(got.cpu().numpy(), want, what=f"gemma3 decode window={window}")


@pytest.mark.usefixtures("merge_mode")
def test_mla_decode_layer(cuda, orc):
    B, H, Dk, Dv, N = 16, 16, 192, 128, 8192
    kq = pkg.quantize(_randn((B, H, N, Dk), 4, cuda))
    vq = pkg.quantize(_randn((B, H, N, Dv), 5, cuda))
    q = _randn((B, H, 1, Dk), 6, cuda)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q, Dk ** -0.5, kv_len, N, out_dtype=torch.float32,
                                mode="decode")
    want = orc.attention(q.float().cpu().numpy(), _q4_bits(kq), _q4_bits(vq), Dk ** -0.5,
                         causal=False)
    assert_close(got.cpu().numpy(), want, what="mla decode")


def _paged_layer(cuda, A, Hkv, D, total_tokens, dtype, seed):
    bt = 256
    spec = pkg.ModelCacheSpec(n_layers=1, n_kv_heads=Hkv, head_dim=D, block_tokens=bt,
                              layer_types=["global"])
    nblocks = sum(-(-n // bt) for n in total_tokens) + 4
    alloc = pkg.shuffled_allocator(spec, nblocks, seed=seed)
    pool = pkg.PagedQ4Pool.for_spec(spec, nblocks, dtype, cuda)
    layer = pkg.PagedLayerCache(pool, alloc, 0, [f"agent{i}" for i in range(A)], max(total_tokens))
    return pool, layer


def test_chunked_prefill_config_shape(cuda, orc):
    A, Hq, Hkv, D, P, L = 2, 32, 8, 128, 4096, 512
    pool, layer = _paged_layer(cuda, A, Hkv, D, [P + L] * A, torch.bfloat16, seed=7)
    layer.append(_randn((A, Hkv, P, D), 8, cuda, torch.bfloat16), _randn((A, Hkv, P, D), 9, cuda, torch.bfloat16))
    layer.append(_randn((A, Hkv, L, D), 10, cuda, torch.bfloat16), _randn((A, Hkv, L, D), 11, cuda, torch.bfloat16))
    q = _randn((A, Hq, L, D), 12, cuda, torch.bfloat16)
    out = torch.empty(A, Hq, L, D, dtype=torch.float32, device=cuda)
    layer.attention(q, D ** -0.5, out=out, mode="prefill")
    want = orc.attention(q.float().cpu().numpy(), _q4_bits(pool.k), _q4_bits(pool.v), D ** -0.5,
                         sdtype=BF16, n_kv_heads=Hkv, layout=1, block_table=layer._table_host.numpy(),
                         kv_len=np.array(layer.lengths), causal=True)
    assert_close(out.cpu().numpy(), want, what="chunked prefill, config shape")


@pytest.mark.usefixtures("merge_mode")
def test_multi_agent_decode_sample(cuda, orc):
    lens = [1024, 32768, 1025, 32767, 9000, 20000]
    A, Hq, Hkv, D = len(lens), 32, 8, 128
    pool, layer = _paged_layer(cuda, A, Hkv, D, [n + 1 for n in lens], torch.float16, seed=11)
    for r, n in enumerate(lens):
        layer.reserve(r, n + 1)
    for r, n in enumerate(lens):
        k = _randn((1, Hkv, n + 1, D), 100 + r, cuda)
        v = _randn((1, Hkv, n + 1, D), 200 + r, cuda)
        pkg.kernels.append(pkg.kernels.paged_view(pool.k, pool.v, layer.table[r:r + 1].contiguous()),
                           k, v, torch.zeros(1, dtype=torch.int32, device=cuda))
    layer.set_lengths([n + 1 for n in lens])
    q = _randn((A, Hq, 1, D), 300, cuda)
    out = torch.empty(A, Hq, 1, D, dtype=torch.float32, device=cuda)
    layer.attention(q, D ** -0.5, out=out, mode="decode")
    want = orc.attention(q.float().cpu().numpy(), _q4_bits(pool.k), _q4_bits(pool.v), D ** -0.5,
                         n_kv_heads=Hkv, layout=1, block_table=layer._table_host.numpy(),
                         kv_len=np.array(layer.lengths), causal=False)
    assert_close(out.cpu().numpy(), want, what="multi-agent decode sample")


@pytest.mark.parametrize("window", [0, 1024], ids=["global", "window1024"])
def test_gemma3_prefill_chunk(cuda, orc, window):
    B, Hq, Hkv, D, N, L = 8, 16, 8, 256, 4096, 512
    kq = pkg.quantize(_randn((B, Hkv, N, D), 21, cuda))
    vq = pkg.quantize(_randn((B, Hkv, N, D), 22, cuda))
    q = _randn((B, Hq, L, D), 23, cuda)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q, D ** -0.5, kv_len, N, causal=True, window=window,
                                out_dtype=torch.float32, mode="prefill")
    want = orc.attention(q.float().cpu().numpy(), _q4_bits(kq), _q4_bits(vq), D ** -0.5,
                         causal=True, window=window)
    assert_close(got.cpu().numpy(), want, what=f"gemma3 prefill window={window}")


def test_mla_prefill_chunk(cuda, orc):
    B, H, Dk, Dv, N, L = 16, 16, 192, 128, 8192, 512
    kq = pkg.quantize(_randn((B, H, N, Dk), 24, cuda))
    vq = pkg.quantize(_randn((B, H, N, Dv), 25, cuda))
    q = _randn((B, H, L, Dk), 26, cuda)
    view, n = pkg.kernels.contiguous_view(kq, vq)
    kv_len = torch.full((B,), N, dtype=torch.int32, device=cuda)
    got = pkg.kernels.attention(view, q, Dk ** -0.5, kv_len, N, causal=True,
                                out_dtype=torch.float32, mode="prefill")
    want = orc.attention(q.float().cpu().numpy(), _q4_bits(kq), _q4_bits(vq), Dk ** -0.5,
                         causal=True)
    assert_close(got.cpu().numpy(), want, what="mla prefill")
