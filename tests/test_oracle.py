"""CPU checks of the oracle itself, against what the reference's own tests pin.

The reference's tests pin: the Q4 dtype rule (bf16 input -> bf16
scales/biases, uint32 codes: tests/mlx/test_real_cache_round_trip.py:329-337), shapes
[..., D/8] / [..., D/64] (tests/mlx/test_fused_attention_gpu.py:36-49), the Q4 byte
formula (tests/unit/test_analytical_estimates.py:92-190), persistence bit-identity
(tests/integration/test_cache_round_trip.py:100-230) and B=1 vs B=2 consistency
(tests/mlx/test_fused_attention_gpu.py:289-310).  No test there pins code or output
values, so the two independent restatements (NumPy and C) are also checked against each
other bit-for-bit, and against the committed golden fixtures.
"""

from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).parent / "golden"


def _f16(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float16)


@pytest.mark.parametrize("shape", [(1, 64), (33, 128), (4, 3, 192), (2, 256)])
def test_numpy_and_c_quantize_agree_f16(orc, shape):
    x = _f16(shape, sum(shape)).view(np.uint16)
    a = orc.quantize_np(x, orc.F16)
    b = orc.quantize(x, orc.F16)
    for p, q in zip(a, b):
        np.testing.assert_array_equal(p, q)


def test_numpy_and_c_quantize_agree_bf16(orc):
    x = orc.f32_to_bf16_bits(np.random.default_rng(1).standard_normal((50, 128)).astype(np.float32) * 3)
    a = orc.quantize_np(x, orc.BF16)
    b = orc.quantize(x, orc.BF16)
    for p, q in zip(a, b):
        np.testing.assert_array_equal(p, q)


def test_dtype_and_shape_rule(orc):
    """uint32 codes [..., D/8]; scales/biases [..., D/64] in the input dtype."""
    x = _f16((1, 4, 32, 64), 0).view(np.uint16)
    c, s, b = orc.quantize(x, orc.F16)
    assert c.dtype == np.uint32 and c.shape == (1, 4, 32, 8)
    assert s.shape == b.shape == (1, 4, 32, 1)
    xb = orc.f32_to_bf16_bits(np.ones((2, 64), np.float32))
    c, s, b = orc.quantize(xb, orc.BF16)
    # bf16 bit patterns (not fp16): 1.0 stored as bias 0x3f80 in bf16
    assert s.dtype == np.uint16 and (b == 0x3F80).all() or (orc.bf16_bits_to_f32(b) + 15 * orc.bf16_bits_to_f32(s) == 1).all()


def test_zero_is_exact_and_error_bound(orc):
    """mlx's affine rule makes the group's dominant endpoint exact and keeps the
    reconstruction within about one step of every value."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((500, 64)).astype(np.float16)
    c, s, b = orc.quantize_np(x.view(np.uint16), orc.F16)
    deq = orc.dequantize_np(c, s, b, orc.F16)
    step = np.abs(orc.to_f32(s, orc.F16))
    err = np.abs(deq - x.astype(np.float32))
    assert (err <= 1.01 * step + 1e-3).all()
    # a group containing 0 reconstructs 0 exactly when q0 != 0
    z = np.linspace(-1, 3, 64).astype(np.float16)
    z[10] = 0
    c, s, b = orc.quantize_np(z[None].view(np.uint16), orc.F16)
    deq = orc.dequantize_np(c, s, b, orc.F16)
    assert deq[0, 10] == pytest.approx(0.0, abs=2e-3)


def test_degenerate_groups(orc):
    x = np.zeros((3, 64), np.float16)
    x[1] = 2.5
    x[2] = -7
    c, s, b = orc.quantize(x.view(np.uint16), orc.F16)
    d = orc.dequantize(c, s, b, orc.F16)
    np.testing.assert_allclose(d, x.astype(np.float32), atol=1e-6)


def test_q4_byte_formula_matches_reference_tests(orc, am):
    """Values pinned by tests/unit/test_analytical_estimates.py:98-117."""
    assert orc.q4_bytes_per_block_per_layer(8, 256, 256) == 589_824
    spec = am.ModelCacheSpec(n_layers=48, n_kv_heads=8, head_dim=256, block_tokens=256,
                             layer_types=["global"] * 48)
    assert spec.bytes_per_block_per_layer() == 589_824
    fp16 = am.ModelCacheSpec(n_layers=48, n_kv_heads=8, head_dim=256, block_tokens=256,
                             layer_types=["global"] * 48, kv_bits=None)
    assert fp16.bytes_per_block_per_layer() == 2_097_152
    r = spec.bytes_per_block_per_layer() / fp16.bytes_per_block_per_layer()
    assert abs(r - 0.28125) < 1e-3
    mla = am.ModelCacheSpec(n_layers=27, n_kv_heads=16, head_dim=192, v_head_dim=128,
                            block_tokens=256, layer_types=["global"] * 27)
    assert mla.bytes_per_block_per_layer() == orc.q4_bytes_per_block_per_layer(16, 192, 256, 128)


@pytest.mark.parametrize("window,lp", [(0, None), (50, None), (0, [0, 7]), (64, [3, 0])])
def test_c_and_numpy_attention_agree(orc, window, lp):
    rng = np.random.default_rng(3)
    B, Hq, Hkv, N, D, L = 2, 6, 2, 300, 128, 3
    k = rng.standard_normal((B, Hkv, N, D)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, N, D)).astype(np.float16)
    kq, vq = orc.quantize(k.view(np.uint16)), orc.quantize(v.view(np.uint16))
    q = rng.standard_normal((B, Hq, L, D)).astype(np.float32)
    kvs = None if lp is None else np.array(lp)
    a = orc.attention(q, kq, vq, 0.1, window=window, kv_start=kvs)
    b = orc.attention_np(q, kq, vq, 0.1, window=window, kv_start=kvs)
    np.testing.assert_allclose(a, b, atol=2e-6, rtol=1e-5)


def test_paged_oracle_matches_contiguous(orc):
    rng = np.random.default_rng(9)
    Hkv, D, bt = 2, 64, 16
    lens = [40, 17]
    k = rng.standard_normal((2, Hkv, 48, D)).astype(np.float16)
    v = rng.standard_normal((2, Hkv, 48, D)).astype(np.float16)
    kq, vq = orc.quantize(k.view(np.uint16)), orc.quantize(v.view(np.uint16))
    table = np.array([[4, 0, 2], [5, 1, -1]], np.int32)
    pk = [np.zeros((6, Hkv, bt) + a.shape[3:], a.dtype) for a in kq]
    pv = [np.zeros((6, Hkv, bt) + a.shape[3:], a.dtype) for a in vq]
    for b in range(2):
        for t in range(lens[b]):
            blk = table[b, t // bt]
            for P, S in ((pk, kq), (pv, vq)):
                for p, s in zip(P, S):
                    p[blk, :, t % bt] = s[b, :, t]
    q = rng.standard_normal((2, 4, 1, D)).astype(np.float32)
    a = orc.attention(q, tuple(pk), tuple(pv), 0.125, n_kv_heads=Hkv, layout=1, block_table=table,
                      kv_len=np.array(lens), causal=False)
    b = orc.attention(q, kq, vq, 0.125, kv_len=np.array(lens), causal=False)
    np.testing.assert_allclose(a, b, atol=1e-6)


def test_batch_split_consistency_oracle(orc):
    rng = np.random.default_rng(11)
    k = rng.standard_normal((2, 2, 100, 64)).astype(np.float16)
    kq = orc.quantize(k.view(np.uint16))
    q = rng.standard_normal((2, 4, 1, 64)).astype(np.float32)
    both = orc.attention(q, kq, kq, 0.1, causal=False)
    one = orc.attention(q[1:], tuple(a[1:] for a in kq), tuple(a[1:] for a in kq), 0.1, causal=False)
    np.testing.assert_allclose(both[1:], one, atol=1e-6)


def test_mlx_fp16_emulation_close_to_fp32(orc):
    """The reference's fp16-intermediate rounding stays within the attention tolerance of
    the fp32 oracle on N(0,1) data (bounds the gap the kernels are measured against)."""
    rng = np.random.default_rng(2)
    B, Hq, Hkv, N, D = 1, 8, 2, 512, 128
    k = rng.standard_normal((B, Hkv, N, D)).astype(np.float16)
    v = rng.standard_normal((B, Hkv, N, D)).astype(np.float16)
    kq, vq = orc.quantize(k.view(np.uint16)), orc.quantize(v.view(np.uint16))
    q = rng.standard_normal((B, Hq, 1, D)).astype(np.float16)
    a = orc.attention_mlx_fp16_np(q, kq, vq, D ** -0.5).astype(np.float32)
    b = orc.attention(q.astype(np.float32), kq, vq, D ** -0.5, causal=False)
    assert np.abs(a - b).max() < 2e-3 + 1e-3 * np.abs(b).max()


@pytest.mark.parametrize("name", sorted(p.name for p in GOLDEN.glob("*.npz")))
def test_golden_fixture(orc, name):
    """Committed fixtures (tests/golden/make_golden.py) reproduce bit-for-bit / to 1e-6."""
    f = np.load(GOLDEN / name)
    kind = str(f["kind"])
    if kind == "quantize":
        got = orc.quantize(f["x"], int(f["dtype"]))
        for g, w in zip(got, (f["codes"], f["scales"], f["biases"])):
            np.testing.assert_array_equal(g, w)
    elif kind == "attention":
        kq = (f["kc"], f["ks"], f["kb"])
        vq = (f["vc"], f["vs"], f["vb"])
        kvs = f["kv_start"] if "kv_start" in f.files else None
        got = orc.attention(f["q"], kq, vq, float(f["scale"]), sdtype=int(f["sdtype"]),
                            causal=bool(f["causal"]), window=int(f["window"]), kv_start=kvs)
        np.testing.assert_allclose(got, f["out"], atol=1e-5, rtol=1e-5)
    elif kind == "ref_sdpa":
        # output of the reference's own patched quantized SDPA (mlx_fused_attention.py), run
        # over the NumPy mlx stand-in: its fp16 intermediates stay within the attention
        # tolerance of the fp32 oracle, which pins the oracle's mask / GQA / op-order rules
        q = f["q"].view(np.float16).astype(np.float32)
        kq = (f["kc"], f["ks"], f["kb"])
        vq = (f["vc"], f["vs"], f["vb"])
        mask, mk, causal = None, 0, False
        if "mask_str" in f.files:
            causal = True
        elif "mask" in f.files:
            mask = f["mask"]
            mk = 1 if mask.dtype == bool else 2
            mask = mask.astype(np.float32)
        got = orc.attention(q, kq, vq, float(f["scale"]), causal=causal, mask=mask, mask_kind=mk)
        ref = f["out"].view(np.float16).astype(np.float32)
        assert np.all(np.abs(got - ref) <= 2e-3 + 1e-3 * np.abs(ref))
    elif kind == "ref_sinks":
        # output of the reference's sink shim (mlx_sink_compat.py: dequantize, then fast SDPA
        # with per-head sink logits) over the stand-in: pins the oracle's sink rule
        q = f["q"].view(np.float16).astype(np.float32)
        kq = (f["kc"], f["ks"], f["kb"])
        vq = (f["vc"], f["vs"], f["vb"])
        mask, mk, causal = None, 0, "mask_str" in f.files
        if "mask" in f.files:
            mask = f["mask"].astype(np.float32)
            mk = 1
        got = orc.attention(q, kq, vq, float(f["scale"]), causal=causal, mask=mask, mask_kind=mk,
                            sinks=f["sinks"])
        ref = f["out"].view(np.float16).astype(np.float32)
        assert np.all(np.abs(got - ref) <= 2e-3 + 1e-3 * np.abs(ref))
        # the sinks matter: without them the outputs differ
        plain = orc.attention(q, kq, vq, float(f["scale"]), causal=causal, mask=mask, mask_kind=mk)
        assert np.abs(plain - ref).max() > 1e-2
    elif kind == "cache_lifecycle":
        # the recorded inputs re-quantized by the oracle reproduce the reference cache's
        # packed codes (the cache bookkeeping itself is replayed on the GPU)
        meta = __import__("json").loads(str(f["meta"]))
        assert [m["tag"] for m in meta][:3] == ["merge", "update1", "update2"]
        c1 = orc.quantize(f["in_c1_k"], orc.F16)
        np.testing.assert_array_equal(f["merge_kc"][0, :, meta[0]["left_padding"][0]:], c1[0][0])
    else:
        pytest.fail(f"unknown fixture kind {kind}")


def test_block_pool_replays_reference(am):
    """tests/golden/ref_block_pool.json: the reference's BlockPool on a fixed op sequence."""
    import json

    log = json.loads((GOLDEN / "ref_block_pool.json").read_text())
    spec = am.ModelCacheSpec(n_layers=4, n_kv_heads=8, head_dim=128, block_tokens=256,
                             layer_types=["global"] * 4)
    pool = am.BlockPool(spec, 32)
    held = {}
    for op in log:
        if op[0] == "alloc":
            got = pool.allocate(len(op[3]), op[2], op[1])
            assert [b.block_id for b in got] == op[3]
            held.setdefault(op[1], []).extend(got)
        elif op[0] == "free":
            blocks = [b for b in held[op[1]] if b.block_id in op[2]]
            pool.free(blocks, op[1])
        elif op[0] == "free_agent":
            assert pool.free_agent_blocks(op[1]) == op[2]
        elif op[0] == "state":
            assert [pool.available_blocks(), pool.allocated_block_count(), pool.used_memory(),
                    pool.max_batch_size(600)] == op[1:]
