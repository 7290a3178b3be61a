"""reshape_and_cache and the KVCache wrapper on the GPU: bit-exact against the
oracle's restatement of src/kv_cache.rs:212-357."""
import numpy as np
import pytest

from helpers import bf16_tensor, f32_tensor

pytestmark = pytest.mark.gpu


# Shapes: 16-byte chunks per token row of 8, 128, 18, 256 (block size 12, not a
# power of two) and 512 on the vector form; 20-byte rows on the element form.
@pytest.mark.parametrize("dtype,Hkv,d,bs", [("f32", 4, 8, 16), ("bf16", 8, 128, 16),
                                            ("bf16", 2, 72, 8), ("bf16", 8, 256, 12),
                                            ("f32", 16, 128, 16), ("f32", 3, 5, 4)])
def test_reshape_and_cache_bit_exact(ctx, oracle, dtype, Hkv, d, bs):
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(Hkv * 100 + d)
    nb, T = 128, 300
    k = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    slots = rng.permutation(nb * bs)[:T].astype(np.int64)
    slots[::17] = -1  # skipped tokens
    if dtype == "bf16":
        (tk, _), (tv, _) = bf16_tensor(oracle, k), bf16_tensor(oracle, v)
        hk, hv = oracle.f32_to_bf16_bits(k), oracle.f32_to_bf16_bits(v)
        pk = np.zeros((nb, Hkv, bs, d), np.uint16)
    else:
        tk, tv, hk, hv = f32_tensor(k), f32_tensor(v), k, v
        pk = np.zeros((nb, Hkv, bs, d), np.float32)
    pv = np.zeros_like(pk)
    gk = torch.zeros((nb, Hkv, bs, d), dtype=tk.dtype, device="cuda")
    gv = torch.zeros_like(gk)
    zb.CudaAttention(ctx).reshape_and_cache(tk, tv, gk, gv, torch.from_numpy(slots).cuda(), Hkv, d, bs, nb)
    ctx.check_status()
    assert oracle.reshape_and_cache(pk, pv, hk, hv, slots, Hkv, d, bs, nb) == 0
    view = (lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)) if dtype == "bf16" else (lambda t: t.cpu().numpy())
    assert np.array_equal(view(gk), pk) and np.array_equal(view(gv), pv)


def test_reshape_and_cache_oob_slot(ctx):
    import torch
    import zealot_b200 as zb
    nb, bs, Hkv, d = 4, 16, 2, 8
    k = torch.randn((3, Hkv, d), device="cuda")
    pool = torch.zeros((nb, Hkv, bs, d), device="cuda")
    slots = torch.tensor([0, nb * bs, 5], dtype=torch.int64, device="cuda")
    zb.CudaAttention(ctx).reshape_and_cache(k, k, pool, pool.clone(), slots, Hkv, d, bs, nb)
    with pytest.raises(zb.OobBlockError):
        ctx.check_status()
    assert torch.equal(pool[0, :, 5], k[2])


def test_reshape_and_cache_c3_round_trip(ctx):
    """Config C3 scale (16 sequences, lengths U[256, 8192], 8 kv heads, d 128, bf16):
    scatter through a seeded random slot mapping, gather back, compare bytes."""
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(33)
    lens = rng.integers(256, 8193, size=16)
    T = int(lens.sum())
    Hkv, d, bs = 8, 128, 16
    nb = (T + bs - 1) // bs + 64
    g = torch.Generator(device="cuda").manual_seed(33)
    k = torch.randn((T, Hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((T, Hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.from_numpy(rng.permutation(nb * bs)[:T].astype(np.int64)).cuda()
    pk = torch.zeros((nb, Hkv, bs, d), dtype=torch.bfloat16, device="cuda")
    pv = torch.zeros_like(pk)
    zb.CudaAttention(ctx).reshape_and_cache(k, v, pk, pv, slots, Hkv, d, bs, nb)
    ctx.check_status()
    blk, off = slots // bs, slots % bs
    back_k = pk[blk, :, off, :]
    back_v = pv[blk, :, off, :]
    assert torch.equal(back_k.view(torch.int16), k.view(torch.int16))
    assert torch.equal(back_v.view(torch.int16), v.view(torch.int16))


def test_kv_cache_store_and_append(ctx, oracle):
    """KVCache::store_kv / append_kv / alloc_block / -1 sentinels (kv_cache.rs:107-357)."""
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(12)
    nb, bs, L, Hkv, d = 32, 16, 2, 4, 8
    bm = zb.BlockManager(nb, bs)
    kv = zb.KVCache(ctx, nb, bs, L, Hkv, d)
    kv.register_seq("a", 8)
    with pytest.raises(zb.InternalError):
        kv.store_kv(0, "zz", 0, 0, 0, 1)  # unknown seq
    handles = [kv.alloc_block("a", bm) for _ in range(3)]
    assert [h.block_id for h in handles] == [0, 1, 2]
    k = rng.standard_normal((40, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((40, Hkv, d)).astype(np.float32)
    kv.store_kv(1, "a", f32_tensor(k), f32_tensor(v), 3, 40)
    with pytest.raises(zb.InternalError):
        kv.store_kv(1, "a", f32_tensor(k), f32_tensor(v), 10, 40)  # block_idx OOB
    one_k = rng.standard_normal((1, Hkv, d)).astype(np.float32)
    kv.append_kv(1, "a", f32_tensor(one_k), f32_tensor(one_k))
    assert kv.cached_tokens("a") == 1  # store_kv does not advance it (kv_cache.rs:212-276)
    torch.cuda.synchronize()
    ref_k = np.zeros((nb, Hkv, bs, d), np.float32)
    ref_v = np.zeros_like(ref_k)
    ids = np.array([h.block_id for h in handles], np.int64)
    oracle.store_kv(ref_k, ref_v, k, v, ids, 3, 40, Hkv, d, bs)
    oracle.store_kv(ref_k, ref_v, one_k, one_k, ids, 0, 1, Hkv, d, bs)  # append lands at token 0
    assert np.array_equal(kv.k_pool(1).cpu().numpy(), ref_k)
    assert np.array_equal(kv.v_pool(1).cpu().numpy(), ref_v)
    assert np.all(kv.k_pool(0).cpu().numpy() == 0)
    assert kv.block_table("a", 8).cpu().tolist() == [0, 1, 2, -1, -1, -1, -1, -1]
    kv.release_seq("a")
    assert kv.block_table_ptr("a") == 0
