"""Paged batch-cache lifecycle (merge / update_and_fetch / filter / extend / extract / trim
as block-table edits), the device free list, and Q4 block persistence.

The contiguous BatchQuantizedKVCache (bit-identical to the reference's own code on the
golden fixtures) is driven through the same operations; after each one the paged cache
must hold the same Q4 codes, scales and biases for every sequence (bit-exact) and give the
same attention outputs (both fp32-accumulating kernels: 2e-3 abs + 1e-3 rel).
"""

import numpy as np
import pytest
import torch

from conftest import assert_close, pkg

pytestmark = pytest.mark.gpu

H, HQ, D, BT = 2, 8, 128, 256
persistence = __import__(pkg.__name__ + ".persistence", fromlist=["persistence"])


def _kv(g, B, L, cuda):
    k = torch.randn(B, H, L, D, generator=g).half().to(cuda)
    v = torch.randn(B, H, L, D, generator=g).half().to(cuda)
    return k, v


def _rows(state, lengths):
    """Per-row valid codes/scales/biases of a right-aligned [B, H, N, .] state."""
    k, v = state[0], state[1]
    N = k[0].shape[2]
    return [[t[r, :, N - L:].cpu() for t in (*k, *v)] for r, L in enumerate(lengths)]


def _contig_rows(c):
    k, v, _, lp = c.state
    N = k[0].shape[2]
    return [[t[r, :, int(lp[r]):N].cpu() for t in (*k, *v)] for r in range(k[0].shape[0])]


def _same_codes(paged, contig):
    a = _rows(paged.state, paged.lengths)
    b = _contig_rows(contig)
    assert len(a) == len(b)
    for ra, rb in zip(a, b):
        for x, y in zip(ra, rb):
            assert x.shape == y.shape and torch.equal(x, y)


def _attend(paged, contig, g, cuda):
    B = paged.rows
    q = torch.randn(B, HQ, 1, D, generator=g).half().to(cuda)
    kp, vp = pkg.PagedKV(paged, "k"), pkg.PagedKV(paged, "v")
    a = pkg.quantized_scaled_dot_product_attention(q, kp, vp, D ** -0.5, paged.make_mask(1))
    ck, cv, _, lp = contig.state
    N = ck[0].shape[2]
    b = pkg.quantized_scaled_dot_product_attention(q, ck, cv, D ** -0.5,
                                                   pkg.CausalMask(1, N - 1, None, lp))
    assert_close(a.float().cpu().numpy(), b.float().cpu().numpy(), what="paged vs contiguous")


def test_lifecycle_matches_contiguous_cache(cuda):
    g = torch.Generator().manual_seed(0)
    pool = pkg.PagedQ4Pool(H, D, D, 64, BT, torch.float16, cuda)
    alloc = pkg.DeviceBlockPool(64, cuda)
    lens = [300, 40, 530]
    singles_p, singles_c = [], []
    for n in lens:
        k, v = _kv(g, 1, n, cuda)
        p = pkg.PagedBatchQuantizedKVCache(pool, alloc, 1, rows=1)
        p.update_and_fetch(k, v)
        c = pkg.QuantizedKVCache()
        c.update_and_fetch(k, v)
        singles_p.append(p)
        singles_c.append(c)
    P = pkg.PagedBatchQuantizedKVCache.merge(singles_p)
    C = pkg.BatchQuantizedKVCache.merge(singles_c)
    _same_codes(P, C)
    # decode steps, one crossing a block boundary (530 -> 535 stays, 300 -> 305 ...)
    for _ in range(5):
        k, v = _kv(g, 3, 1, cuda)
        P.update_and_fetch(k, v)
        C.update_and_fetch(k, v)
    alloc.check()
    _same_codes(P, C)
    _attend(P, C, g, cuda)
    # filter: keep rows 2 and 0 (row 1's block goes back to the free list)
    free_before = alloc.available_blocks()
    P.filter([2, 0])
    C.filter([2, 0])
    assert alloc.available_blocks() == free_before + 1
    _same_codes(P, C)
    for _ in range(2):
        k, v = _kv(g, 2, 1, cuda)
        P.update_and_fetch(k, v)
        C.update_and_fetch(k, v)
    _attend(P, C, g, cuda)
    # extend with a new sequence of 100 tokens
    k, v = _kv(g, 1, 100, cuda)
    p1 = pkg.PagedBatchQuantizedKVCache(pool, alloc, 1, rows=1)
    p1.update_and_fetch(k, v)
    c1 = pkg.QuantizedKVCache()
    c1.update_and_fetch(k, v)
    P.extend(p1)
    C.extend(pkg.BatchQuantizedKVCache.merge([c1]))
    _same_codes(P, C)
    k, v = _kv(g, 3, 1, cuda)
    P.update_and_fetch(k, v)
    C.update_and_fetch(k, v)
    _attend(P, C, g, cuda)
    # trim 3 tokens from every row
    assert P.trim(3) == C.trim(3) == 3
    _same_codes(P, C)
    _attend(P, C, g, cuda)
    # extract row 1 as a single-sequence cache
    e_p = P.extract(1)
    e_c = C.extract(1)
    a = _rows(e_p.state, e_p.lengths)[0]
    b = [t[0].cpu() for t in (*e_c.keys, *e_c.values)]
    for x, y in zip(a, b):
        assert torch.equal(x, y[:, :x.shape[1]]) and x.shape[1] == e_c.offset
    # every block is accounted for
    used = sum(-(-n // BT) for n in P.lengths) + sum(-(-n // BT) for n in e_p.lengths)
    assert alloc.available_blocks() + used == 64
    P.free()
    e_p.free()
    assert alloc.available_blocks() == 64
    alloc.check()


def test_device_free_list_matches_block_pool(cuda):
    """Reserve / release on the device hand out and take back the ids the host BlockPool
    (services.py:111-223) does for the same calls."""
    spec = pkg.ModelCacheSpec(n_layers=1, n_kv_heads=H, head_dim=D, block_tokens=BT,
                              layer_types=["global"])
    host = pkg.BlockPool(spec, 12)
    dev = pkg.DeviceBlockPool.from_host(host, cuda)
    table = torch.full((3, 6), -1, dtype=torch.int32, device=cuda)
    lengths = torch.zeros(3, dtype=torch.int32, device=cuda)
    add = torch.tensor([600, 10, 1100], dtype=torch.int32, device=cuda)
    dev.reserve(table, lengths, add, BT)
    dev.check()
    expect = []
    for n in (600, 10, 1100):
        expect.append([b.block_id for b in host.allocate(-(-n // BT), 0, "a")])
    t = table.cpu().tolist()
    for r, ids in enumerate(expect):
        assert t[r][:len(ids)] == ids and all(x == -1 for x in t[r][len(ids):])
    assert dev.free_list() == host.free_list
    # release: row 0 keeps 1 block, row 2 keeps none
    keep = torch.tensor([1, 6, 0], dtype=torch.int32, device=cuda)
    dev.release(table, keep)
    dev.check()
    for bid in expect[0][1:] + expect[2]:
        host.free([host.allocated_blocks[bid]], "a")
    assert dev.free_list() == host.free_list
    # exhaustion (16 missing entries, 10 free): all-or-nothing, state unchanged, and
    # PoolExhaustedError on check()
    before = (table.clone(), dev.available_blocks())
    dev.reserve(table, torch.zeros(3, dtype=torch.int32, device=cuda),
                torch.full((3,), 6 * BT, dtype=torch.int32, device=cuda), BT)
    with pytest.raises(pkg.PoolExhaustedError):
        dev.check()
    assert torch.equal(table, before[0]) and dev.available_blocks() == before[1]


def test_persistence_round_trip_through_pool_blocks(cuda, tmp_path):
    g = torch.Generator().manual_seed(3)
    pool = pkg.PagedQ4Pool(H, D, D, 32, BT, torch.float16, cuda)
    alloc = pkg.DeviceBlockPool(32, cuda)
    P = pkg.PagedBatchQuantizedKVCache(pool, alloc, 1, rows=1)
    k, v = _kv(g, 1, 700, cuda)
    P.update_and_fetch(k, v)
    n = P.lengths[0]
    ids = P.table[0, :-(-n // BT)].tolist()
    layers = {0: [(bid, min(BT, n - i * BT)) for i, bid in enumerate(ids)]}
    path = persistence.save_blocks(tmp_path / "a1.safetensors", pool, layers, {"n": n})
    # load into a second pool at other block ids
    pool2 = pkg.PagedQ4Pool(H, D, D, 32, BT, torch.float16, cuda)
    spec = pkg.ModelCacheSpec(n_layers=1, n_kv_heads=H, head_dim=D, block_tokens=BT,
                              layer_types=["global"])
    host = pkg.BlockPool(spec, 32)
    store = persistence.SafetensorsQ4Store(tmp_path, pool2, host)
    blocks, meta = store.load(path, "a1")
    assert meta == {"n": str(n)}
    new_ids = [b.block_id for b in blocks[0]]
    assert [b.token_count for b in blocks[0]] == [BT, BT, n - 2 * BT]
    for t1, t2 in zip((*pool.k, *pool.v), (*pool2.k, *pool2.v)):
        for i, (a, b) in enumerate(zip(ids, new_ids)):
            T = min(BT, n - i * BT)
            assert torch.equal(t1[a, :, :T], t2[b, :, :T])
    # the reference's own file layout: tensors [1, H, T, cols] readable by safetensors
    from safetensors import safe_open

    cq = pkg.quantize(k)
    cv = pkg.quantize(v)
    with safe_open(str(path), framework="numpy") as f:
        for i in range(len(ids)):
            T = min(BT, n - i * BT)
            sl = slice(i * BT, i * BT + T)
            w = f.get_tensor(f"L0_B{i}_K_weights")
            assert w.dtype == np.uint32 and w.shape == (1, H, T, D // 8)
            assert np.array_equal(w[0], cq[0][0, :, sl].cpu().numpy().view(np.uint32))
            assert np.array_equal(f.get_tensor(f"L0_B{i}_V_biases")[0],
                                  cv[2][0, :, sl].cpu().numpy())


def test_load_reference_layout_file(cuda, tmp_path):
    """A file laid out as the reference's save() writes it (one [1, H, T, cols] tensor per
    block part) loads into pool blocks; attention over them equals the contiguous path."""
    from safetensors.numpy import save_file

    g = torch.Generator().manual_seed(9)
    n = 520
    k, v = _kv(g, 1, n, cuda)
    kq, vq = pkg.quantize(k), pkg.quantize(v)
    tensors = {}
    for i in range(-(-n // BT)):
        sl = slice(i * BT, min(n, (i + 1) * BT))
        for part, q in (("K", kq), ("V", vq)):
            tensors[f"L0_B{i}_{part}_weights"] = q[0][:, :, sl].cpu().numpy().view(np.uint32)
            tensors[f"L0_B{i}_{part}_scales"] = q[1][:, :, sl].cpu().numpy()
            tensors[f"L0_B{i}_{part}_biases"] = q[2][:, :, sl].cpu().numpy()
    path = tmp_path / "ref_agent.safetensors"
    save_file(tensors, str(path), metadata={"model_id": "m"})
    pool = pkg.PagedQ4Pool(H, D, D, 16, BT, torch.float16, cuda)
    spec = pkg.ModelCacheSpec(n_layers=1, n_kv_heads=H, head_dim=D, block_tokens=BT,
                              layer_types=["global"])
    store = persistence.SafetensorsQ4Store(tmp_path, pool, pkg.BlockPool(spec, 16))
    blocks, meta = store.load(path)
    ids = [b.block_id for b in blocks[0]]
    table = torch.tensor([ids], dtype=torch.int32, device=cuda)
    q = torch.randn(1, HQ, 1, D, generator=g).half().to(cuda)
    kv_len = torch.tensor([n], dtype=torch.int32, device=cuda)
    a = pkg.kernels.attention(pool.view(table), q, D ** -0.5, kv_len, n)
    b = pkg.quantized_scaled_dot_product_attention(q, kq, vq, D ** -0.5, None)
    assert_close(a.float().cpu().numpy(), b.float().cpu().numpy(), what="loaded reference file")


def test_engine_glue_extract_save_load_reconstruct(cuda, tmp_path):
    """_extract_cache -> save -> load -> _reconstruct_cache -> _slice_cache_to_length
    (batch_engine.py:1690-2064) over pool blocks: the agent's blocks never leave the pool
    except through the file, and attention after the round trip is unchanged."""
    g = torch.Generator().manual_seed(11)
    layers, n = 2, 650
    pool = pkg.PagedQ4Pool(H, D, D, 40, BT, torch.float16, cuda)
    alloc = pkg.DeviceBlockPool(40, cuda)
    kv = [_kv(g, 1, n, cuda) for _ in range(layers)]
    caches = []
    for k, v in kv:
        c = pkg.PagedBatchQuantizedKVCache(pool, alloc, 1, rows=1)
        c.update_and_fetch(k, v)
        caches.append(c)
    q = torch.randn(1, HQ, 1, D, generator=g).half().to(cuda)

    def attend(cs):
        return [pkg.quantized_scaled_dot_product_attention(q, pkg.PagedKV(c, "k"), pkg.PagedKV(c, "v"),
                                                           D ** -0.5, None).float().cpu()
                for c in cs]

    before = attend(caches)
    blocks = pkg.extract_agent_blocks("agent_7", caches, token_sequence=list(range(n)))
    assert blocks.total_tokens == n and [b.token_count for b in blocks.blocks[0]] == [256, 256, 138]
    store = persistence.SafetensorsQ4Store(tmp_path, pool, alloc)
    path = store.save("agent_7", blocks, {"block_tokens": BT})
    for c in caches:
        c.free()
    assert alloc.available_blocks() == 40
    loaded, _ = store.load(path)
    agent = pkg.AgentBlocks(agent_id="agent_7", blocks=loaded, total_tokens=n)
    rebuilt = pkg.reconstruct_cache(agent, pool, alloc, layers)
    for a, b in zip(before, attend(rebuilt)):
        assert torch.equal(a, b)
    # warm hit: keep a 300-token prefix (EXACT-match shortcut + slice to length)
    for c in rebuilt:
        c.free()
    loaded, _ = store.load(path)
    agent = pkg.AgentBlocks(agent_id="agent_7", blocks=loaded, total_tokens=n)
    pref = pkg.reconstruct_cache(agent, pool, alloc, layers, max_tokens=300)
    assert [c.lengths[0] for c in pref] == [512, 512]  # whole blocks up to >= 300 tokens
    assert alloc.available_blocks() == 40 - 2 * 2
    pkg.slice_cache_to_length(pref, 300)
    assert alloc.available_blocks() == 40 - 2 * 2 and [c.lengths[0] for c in pref] == [300, 300]
    got = attend(pref)
    for (k, v), a in zip(kv, got):
        kq, vq = pkg.quantize(k[:, :, :300]), pkg.quantize(v[:, :, :300])
        want = pkg.quantized_scaled_dot_product_attention(q, kq, vq, D ** -0.5, None).float().cpu()
        assert_close(a.numpy(), want.numpy(), what="prefix after slice")
