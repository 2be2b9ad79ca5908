"""CPU tests of the host-side logic: block pool accounting (mirrors the reference's
tests/unit block-pool tests), structured masks vs mlx-lm's create_causal_mask rule, and
the agent partition used for multi-GPU sharding."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import pkg

bp = pkg.block_pool


def spec(layers=4, heads=8, dim=128, window=None):
    types = ["global"] * layers if window is None else ["sliding_window"] * layers
    return pkg.ModelCacheSpec(n_layers=layers, n_kv_heads=heads, head_dim=dim, block_tokens=256,
                              layer_types=types, sliding_window_size=window)


def test_allocate_free_roundtrip():
    pool = pkg.BlockPool(spec(), 100)
    blocks = pool.allocate(4, 0, "a")
    assert pool.available_blocks() == 96 and len(blocks) == 4
    assert all(b.token_count == 0 and b.layer_id == 0 for b in blocks)
    pool.free(blocks, "a")
    assert pool.available_blocks() == 100
    assert pool.used_memory() + pool.available_memory() == pool.total_memory()


def test_exhaustion_leaves_state_unchanged():
    pool = pkg.BlockPool(spec(), 10)
    pool.allocate(8, 1, "a")
    with pytest.raises(pkg.PoolExhaustedError):
        pool.allocate(3, 1, "b")
    assert pool.available_blocks() == 2 and "b" not in pool.agent_allocations


def test_double_free_and_foreign_free_rejected():
    pool = pkg.BlockPool(spec(), 10)
    blocks = pool.allocate(2, 0, "a")
    with pytest.raises(bp.BlockOperationError):
        pool.free(blocks, "b")
    pool.free(blocks, "a")
    with pytest.raises(bp.BlockOperationError):
        pool.free(blocks, "a")


def test_free_agent_blocks_and_reconfigure():
    pool = pkg.BlockPool(spec(), 50)
    pool.allocate(5, 0, "a")
    pool.allocate(3, 2, "a")
    with pytest.raises(bp.PoolConfigurationError):
        pool.reconfigure(spec(layers=8))
    assert pool.free_agent_blocks("a") == 8
    pool.reconfigure(spec(layers=8))
    assert pool.available_blocks() == 50 and pool.spec.n_layers == 8


def test_spec_validation_and_window_blocks():
    with pytest.raises(bp.ModelSpecValidationError):
        pkg.ModelCacheSpec(n_layers=2, n_kv_heads=8, head_dim=128, block_tokens=256,
                           layer_types=["global"])
    with pytest.raises(bp.ModelSpecValidationError):
        pkg.ModelCacheSpec(n_layers=1, n_kv_heads=8, head_dim=128, block_tokens=256,
                           layer_types=["global"], kv_group_size=48)
    s = spec(window=1024)
    assert s.max_blocks_for_layer("sliding_window") == 4
    assert s.max_blocks_for_layer("global") is None
    assert pkg.BlockPool(s, 1000).max_batch_size(512) == 1000 // (2 * 4)


def test_shuffled_allocator_is_a_seeded_permutation():
    a = pkg.shuffled_allocator(spec(), 64, seed=3)
    b = pkg.shuffled_allocator(spec(), 64, seed=3)
    assert a.free_list == b.free_list and sorted(a.free_list) == list(range(64))
    assert a.free_list != list(range(64))


@pytest.mark.parametrize("N,offset,window,lp", [(1, 99, None, None), (5, 20, 8, None),
                                                 (3, 10, None, [0, 4]), (4, 30, 6, [2, 0, 9])])
def test_causal_mask_rule(orc, N, offset, window, lp):
    lpt = None if lp is None else torch.tensor(lp)
    m = pkg.create_causal_mask(N, offset, window, left_padding=lpt)
    cm = pkg.CausalMask(N, offset, window, lpt).to_dense()
    assert torch.equal(m, cm)
    n = offset + N
    for b in range(1 if lp is None else len(lp)):
        keep = orc.structured_keep(n, N, 0 if lp is None else lp[b], True, window or 0)
        got = m if lp is None else m[b, 0]
        assert np.array_equal(got.numpy(), keep)


def test_single_sequence_make_mask_semantics():
    c = pkg.QuantizedKVCache()
    c.offset = 100
    assert c.make_mask(N=1) is None
    assert c.make_mask(N=4) == "causal"
    assert isinstance(c.make_mask(N=4, return_array=True), pkg.CausalMask)
    assert c.make_mask(N=1, window_size=128) is None       # offset <= window
    assert c.make_mask(N=1, window_size=64) is not None
    assert pkg.validate_q4_pipeline()


def test_lpt_partition_balanced_and_complete():
    rng = np.random.default_rng(0)
    lens = rng.integers(1024, 32769, size=256).tolist()
    for world in (1, 2, 4, 8):
        parts = pkg.lpt_partition(lens, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(256))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) / (sum(lens) / world) < 1.01


def test_patch_installer_idempotent_and_env_flag(monkeypatch):
    import types

    mod = types.SimpleNamespace(quantized_scaled_dot_product_attention="orig")
    monkeypatch.setenv("SEMANTIC_DISABLE_FUSED_ATTN", "1")
    assert pkg.apply_fused_attention_patch(mod) is False
    assert mod.quantized_scaled_dot_product_attention == "orig"
    monkeypatch.delenv("SEMANTIC_DISABLE_FUSED_ATTN")
    assert pkg.apply_fused_attention_patch(mod) is True
    assert pkg.apply_fused_attention_patch(mod) is True
    assert mod.quantized_scaled_dot_product_attention is pkg.quantized_scaled_dot_product_attention
    assert mod._original_quantized_sdpa == "orig"


def test_group_size_other_than_64_raises():
    with pytest.raises(NotImplementedError):
        pkg.quantized_scaled_dot_product_attention(None, None, None, 1.0, None, group_size=32)


def _prefill_desc_args(k_dim, v_dim, hkv, hq, batch, q_len, max_kv_len, window=0):
    d = pkg._lib.Q4CacheDesc()
    d.k_codes = d.k_scales = d.k_biases = d.v_codes = d.v_scales = d.v_biases = 4096
    d.scale_dtype, d.layout, d.n_kv_heads, d.k_dim, d.v_dim = 0, 0, hkv, k_dim, v_dim
    d.capacity, d.batch = (max_kv_len + 15) // 16 * 16, batch
    a = pkg._lib.AttnArgs()
    a.q, a.out, a.kv_len = 4096, 4096, 4096
    a.batch, a.n_q_heads, a.q_len, a.max_kv_len, a.window, a.scale = batch, hq, q_len, max_kv_len, window, 0.1
    return d, a


@pytest.mark.parametrize("dims", [(128, 128), (256, 256), (192, 128), (64, 64), (128, 64)])
def test_prefill_workspace_sizing(dims):
    """The prefill workspace holds fp16 rows of every key the block can see, per (sequence,
    KV head): max_kv_len keys, or window + q_len - 1 with a sliding window; K rows first,
    V rows after them on a 256-byte boundary -- except for MLA's K192 / V128, whose
    attention kernel dequantizes V itself (K rows only).  am_q4_attention sizes for the
    kernel it dispatches to."""
    lib = pkg._lib.load()
    dk, dv = dims
    v_rows = (dk, dv) != (192, 128)
    d, a = _prefill_desc_args(dk, dv, 8, 32, 2, 512, 4608)
    want = 2 * 8 * 4608 * (dk + (dv if v_rows else 0)) * 2
    assert lib.am_q4_prefill_workspace_bytes(ctypes.byref(d), ctypes.byref(a)) == want
    assert lib.am_q4_attention_workspace_bytes(ctypes.byref(d), ctypes.byref(a)) == want
    a.window = 1024  # window + q_len - 1 = 1535 keys, rounded up to 1536 rows
    rows = 2 * 8 * 1536
    k_bytes = (rows * dk * 2 + 255) // 256 * 256
    assert lib.am_q4_prefill_workspace_bytes(ctypes.byref(d), ctypes.byref(a)) == \
        k_bytes + (rows * dv * 2 if v_rows else 0)
    a.q_len = 1  # decode-shaped: am_q4_attention takes the split-KV kernel
    assert lib.am_q4_attention_workspace_bytes(ctypes.byref(d), ctypes.byref(a)) == \
        lib.am_q4_decode_workspace_bytes(ctypes.byref(d), ctypes.byref(a))


def test_prefill_without_workspace_is_refused_before_any_launch():
    lib = pkg._lib.load()
    d, a = _prefill_desc_args(128, 128, 8, 32, 2, 512, 4608)
    rc = lib.am_q4_prefill(ctypes.byref(d), ctypes.byref(a), None, 0, None)
    assert rc == pkg._lib.AM_ERR_WORKSPACE
    assert b"workspace" in lib.am_last_error()
    rc = lib.am_q4_prefill(ctypes.byref(d), ctypes.byref(a), 4096 + 128, 1 << 30, None)  # misaligned
    assert rc == pkg._lib.AM_ERR_WORKSPACE
    d.k_dim = d.v_dim = 320
    assert lib.am_q4_prefill(ctypes.byref(d), ctypes.byref(a), None, 0, None) == pkg._lib.AM_ERR_UNSUPPORTED
