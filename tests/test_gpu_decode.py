"""Paged decode on the GPU against the CPU oracle (src/attention/mod.rs:64-97 row math
over the block-table gather of paged_attention.cu). bf16: <= 2e-2 absolute after
softmax, oracle fed the bf16-rounded inputs; fp32: <= 1e-4 relative."""
import numpy as np
import pytest

from helpers import bf16_tensor, decode_case, f32_tensor, rel_err, to_f32

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2
F32_RTOL = 1e-4


def _run_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs, gqa_map=0):
    import torch
    import zealot_b200 as zb
    attn = zb.CudaAttention(ctx)
    tq, q32 = bf16_tensor(oracle, q)
    tk, k32 = bf16_tensor(oracle, kp)
    tv, v32 = bf16_tensor(oracle, vp)
    tt = torch.from_numpy(table).cuda()
    tl = torch.from_numpy(np.asarray(lens, np.int32)).cuda()
    out = torch.full_like(tq, float("nan"))
    B = table.shape[0]
    attn.paged_forward(tq, tk, tv, tt, tl, out, B, H, Hkv, d, bs, table.shape[1],
                       num_blocks=kp.shape[0], gqa_map=gqa_map)
    ctx.check_status()
    ref = oracle.paged_decode(q32, k32, v32, table, lens, H, Hkv, d, bs, kp.shape[0],
                              gqa_map=gqa_map, num_threads=8)
    return to_f32(out), ref


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_bf16_fast_path_small(ctx, oracle, G):
    rng = np.random.default_rng(100 + G)
    Hkv, d, bs = 2, 128, 16
    H = Hkv * G
    lens = [1, 15, 16, 17, 33, 100, 257, 511]
    q, kp, vp, table, lens = decode_case(rng, len(lens), lens, H, Hkv, d, bs, 512)
    got, ref = _run_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs)
    assert np.max(np.abs(got - ref)) <= BF16_ATOL


def test_bf16_empty_and_sentinel(ctx, oracle):
    rng = np.random.default_rng(5)
    H, Hkv, d, bs = 8, 2, 128, 16
    lens = [0, 40, 200, 64]
    q, kp, vp, table, lens = decode_case(rng, 4, lens, H, Hkv, d, bs, 256)
    table[2, 5] = -1  # ends sequence 2 after 80 tokens (paged_attention.cu:66-67)
    got, ref = _run_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs)
    assert np.all(got[0] == 0)
    assert np.max(np.abs(got - ref)) <= BF16_ATOL


def test_bf16_long_context_split(ctx, oracle):
    """Sequences far longer than one warp's share: the stream-K split and the
    last-arriver merge run for almost every (sequence, kv head)."""
    rng = np.random.default_rng(6)
    H, Hkv, d, bs = 32, 8, 128, 16
    lens = [60000, 3000, 17, 20001]
    q, kp, vp, table, lens = decode_case(rng, 4, lens, H, Hkv, d, bs, 6000)
    for _ in range(2):  # twice: the workspace counters must come back to zero
        got, ref = _run_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs)
        assert np.max(np.abs(got - ref)) <= BF16_ATOL


def test_bf16_ragged_many_segments(ctx, oracle):
    """Short and mid-length sequences mixed (48 sequences, 1 to 2600 tokens): most warp
    ranges cross several (sequence, kv head) segments, whole ones and split ones; one
    sequence ends early at a negative table entry."""
    rng = np.random.default_rng(8)
    H, Hkv, d, bs = 32, 8, 128, 16
    lens = np.concatenate([rng.integers(1, 48, size=24), rng.integers(200, 2600, size=24)])
    rng.shuffle(lens)
    nblk = int(((lens + bs - 1) // bs).sum())
    q, kp, vp, table, lens = decode_case(rng, len(lens), lens, H, Hkv, d, bs, nblk + 16)
    table[int(np.argmax(lens)), 3] = -1
    for _ in range(2):  # twice: the workspace counters must come back to zero
        got, ref = _run_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs)
        assert np.max(np.abs(got - ref)) <= BF16_ATOL


def test_bf16_repeatable_across_launches(ctx, oracle):
    """Long ragged ranges (about 30 blocks per warp, most segments split over warps),
    sentinels at several depths, empty sequences, five launches in a row: the merge
    order is fixed by the flat split, so every launch gives the same bytes, and the
    merge counters come back to zero each time."""
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(77)
    H, Hkv, d, bs = 32, 8, 128, 16
    lens = rng.integers(1500, 4000, size=16).astype(np.int64)
    lens[[3, 11]] = 0
    nblk = int(((lens + bs - 1) // bs).sum())
    q, kp, vp, table, lens = decode_case(rng, len(lens), lens, H, Hkv, d, bs, nblk + 16)
    table[5, 40] = -1
    table[9, 2] = -1
    table[13, 150] = -1
    attn = zb.CudaAttention(ctx)
    tq, q32 = bf16_tensor(oracle, q)
    tk, k32 = bf16_tensor(oracle, kp)
    tv, v32 = bf16_tensor(oracle, vp)
    tt = torch.from_numpy(table).cuda()
    tl = torch.from_numpy(np.asarray(lens, np.int32)).cuda()
    ref = oracle.paged_decode(q32, k32, v32, table, lens, H, Hkv, d, bs, kp.shape[0], num_threads=8)
    outs = []
    for _ in range(5):
        out = torch.full_like(tq, float("nan"))
        attn.paged_forward(tq, tk, tv, tt, tl, out, len(lens), H, Hkv, d, bs, table.shape[1],
                           num_blocks=kp.shape[0])
        ctx.check_status()
        got = to_f32(out)
        assert np.max(np.abs(got - ref)) <= BF16_ATOL
        outs.append(got)
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])
    assert np.all(outs[0][3] == 0) and np.all(outs[0][11] == 0)


def test_bf16_c2_full(ctx, oracle):
    """Config C2 at full size: B=64, 32/8 heads, d=128, ctx U[512, 4096], block tables a
    seeded random permutation of a 65536-block pool. The pools are drawn on the GPU; the
    oracle gets the referenced blocks only, with the tables renumbered."""
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(2024)
    B, H, Hkv, d, bs, nb = 64, 32, 8, 128, 16, 65536
    lens = rng.integers(512, 4097, size=B).astype(np.int32)
    nblk = (lens + bs - 1) // bs
    perm = rng.permutation(nb).astype(np.int32)
    table = np.full((B, 256), -1, np.int32)
    off = 0
    for b in range(B):
        table[b, : nblk[b]] = perm[off: off + nblk[b]]
        off += nblk[b]
    g = torch.Generator(device="cuda").manual_seed(2024)
    tk = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    tv = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    tq, q32 = bf16_tensor(oracle, rng.standard_normal((B, H, d)).astype(np.float32))
    out = torch.empty_like(tq)
    attn = zb.CudaAttention(ctx)
    attn.paged_forward(tq, tk, tv, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(),
                       out, B, H, Hkv, d, bs, 256, num_blocks=nb)
    ctx.check_status()
    used = perm[:off]
    idx = torch.from_numpy(used.astype(np.int64)).cuda()
    k32 = tk.index_select(0, idx).float().cpu().numpy()
    v32 = tv.index_select(0, idx).float().cpu().numpy()
    remap = np.full(nb, -1, np.int64)
    remap[used] = np.arange(used.size)
    t2 = np.where(table >= 0, remap[np.maximum(table, 0)], -1).astype(np.int32)
    ref = oracle.paged_decode(q32, k32, v32, t2, lens, H, Hkv, d, bs, used.size, num_threads=8)
    assert np.max(np.abs(to_f32(out) - ref)) <= BF16_ATOL


def test_bf16_modulo_mapping(ctx, oracle):
    rng = np.random.default_rng(8)
    H, Hkv, d, bs = 8, 2, 128, 16
    q, kp, vp, table, lens = decode_case(rng, 3, [30, 99, 160], H, Hkv, d, bs, 64)
    got, ref = _run_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs, gqa_map=1)
    assert np.max(np.abs(got - ref)) <= BF16_ATOL


@pytest.mark.parametrize("shape", [(4, 4, 8, 16), (8, 2, 64, 16), (4, 1, 32, 8)])
def test_f32_generic(ctx, oracle, shape):
    import torch
    import zealot_b200 as zb
    H, Hkv, d, bs = shape
    rng = np.random.default_rng(sum(shape))
    q, kp, vp, table, lens = decode_case(rng, 5, [1, 7, 64, 65, 300], H, Hkv, d, bs, 128)
    attn = zb.CudaAttention(ctx)
    out = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    attn.paged_forward(f32_tensor(q), f32_tensor(kp), f32_tensor(vp), torch.from_numpy(table).cuda(),
                       torch.from_numpy(lens).cuda(), out, 5, H, Hkv, d, bs, table.shape[1])
    ctx.check_status()
    ref = oracle.paged_decode(q, kp, vp, table, lens, H, Hkv, d, bs, kp.shape[0])
    for b in range(5):
        assert rel_err(out[b].cpu().numpy(), ref[b]) <= F32_RTOL


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_oob_block_id_is_reported(ctx, oracle, dtype):
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(9)
    H, Hkv, d, bs = 4, 2, 128, 16
    q, kp, vp, table, lens = decode_case(rng, 2, [40, 40], H, Hkv, d, bs, 32)
    table[1, 1] = 32  # == num_blocks
    with pytest.raises(oracle.OracleError):
        oracle.paged_decode(q, kp, vp, table, lens, H, Hkv, d, bs, 32)
    attn = zb.CudaAttention(ctx)
    if dtype == "bf16":
        tq, tk, tv = (bf16_tensor(oracle, x)[0] for x in (q, kp, vp))
    else:
        tq, tk, tv = f32_tensor(q), f32_tensor(kp), f32_tensor(vp)
    out = torch.empty_like(tq)
    attn.paged_forward(tq, tk, tv, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), out,
                       2, H, Hkv, d, bs, table.shape[1], num_blocks=32)
    with pytest.raises(zb.OobBlockError):
        ctx.check_status()
    ctx.check_status()  # the status word was cleared by the first read


def _check_triple(m, l, o, rm, rl, ro, bf16):
    """Partial triple against the oracle. m is the true maximum score, so it
    matches to fp32 rounding; l sums fp32 probabilities; o is compared after
    normalisation (o / l), with the bf16 tolerance on the bf16 path where the
    probabilities enter the P.V product rounded to bf16."""
    np.testing.assert_allclose(m, rm, rtol=0, atol=1e-4)
    np.testing.assert_allclose(l, rl, rtol=1e-4, atol=1e-30)
    empty = rl == 0
    assert np.all(o[empty] == 0) and np.all(np.isneginf(m[empty]))
    den = np.where(empty, 1.0, rl)[..., None]
    err = float(np.max(np.abs(o / np.where(empty, 1.0, l)[..., None] - ro / den)))
    assert err <= (BF16_ATOL if bf16 else F32_RTOL), err


def _partial_ranges(ctx, oracle, q, kp, vp, table, lens, cuts, H, Hkv, d, bs, dtype):
    """Runs paged_forward_partial over consecutive ranges [cuts[i], cuts[i+1]) of every
    sequence, checks each triple against the oracle and returns the merged output."""
    import torch
    import zealot_b200 as zb
    attn = zb.CudaAttention(ctx)
    bf16 = dtype == "bf16"
    if bf16:
        tq, q32 = bf16_tensor(oracle, q)
        tk, k32 = bf16_tensor(oracle, kp)
        tv, v32 = bf16_tensor(oracle, vp)
    else:
        (tq, tk, tv), (q32, k32, v32) = (f32_tensor(q), f32_tensor(kp), f32_tensor(vp)), (q, kp, vp)
    tt = torch.from_numpy(table).cuda()
    B = table.shape[0]
    ms, ls, os_ = [], [], []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        lo, hi = np.asarray(lo, np.int32), np.asarray(hi, np.int32)
        m = torch.full((B, H), float("nan"), dtype=torch.float32, device="cuda")
        l = torch.full_like(m, float("nan"))
        o = torch.full((B, H, d), float("nan"), dtype=torch.float32, device="cuda")
        attn.paged_forward_partial(tq, tk, tv, tt, torch.from_numpy(lo).cuda(), torch.from_numpy(hi).cuda(),
                                   m, l, o, B, H, Hkv, d, bs, table.shape[1], num_blocks=kp.shape[0])
        ctx.check_status()
        rm, rl, ro = oracle.paged_decode_partial(q32, k32, v32, table, lo, hi, H, Hkv, d, bs, kp.shape[0])
        _check_triple(m.cpu().numpy(), l.cpu().numpy(), o.cpu().numpy(), rm, rl, ro, bf16)
        ms.append(m); ls.append(l); os_.append(o)
    out = torch.empty((B, H, d), dtype=torch.float32, device="cuda")
    attn.merge_partials(torch.stack(ms), torch.stack(ls), torch.stack(os_), out)
    ctx.check_status()
    full = oracle.paged_decode(q32, k32, v32, table, lens, H, Hkv, d, bs, kp.shape[0], num_threads=8)
    return out.cpu().numpy(), full


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_partial_and_merge(ctx, oracle, dtype):
    """Sequence split: partial triples over two token ranges merge to the full decode.
    bf16 runs the fast kernel's partial form, fp32 the CUDA-core kernel."""
    rng = np.random.default_rng(10)
    B, H, Hkv, d, bs = 4, 8, 2, 128, 16
    q, kp, vp, table, lens = decode_case(rng, B, [50, 300, 16, 1000], H, Hkv, d, bs, 256)
    cut = np.array([20, 150, 0, 999], np.int32)
    got, full = _partial_ranges(ctx, oracle, q, kp, vp, table, lens, [np.zeros(B, np.int32), cut, lens],
                                H, Hkv, d, bs, dtype)
    if dtype == "f32":
        assert rel_err(got, full) <= F32_RTOL
    else:
        assert np.max(np.abs(got - full)) <= BF16_ATOL


def test_bf16_partial_ragged_ranges(ctx, oracle):
    """Partial form of the fast kernel: range starts inside a block, empty ranges,
    ranges past a sentinel, sequences long enough that each range splits over many
    warps (last-arriver merge) -- three ranges per sequence merged back."""
    rng = np.random.default_rng(21)
    B, H, Hkv, d, bs = 7, 32, 8, 128, 16
    lens = np.array([0, 5, 300, 1000, 17001, 40000, 2600], np.int32)
    q, kp, vp, table, lens = decode_case(rng, B, lens, H, Hkv, d, bs, 4096)
    table[6, 100] = -1  # sequence 6 ends after 1600 tokens
    c1 = np.array([0, 3, 7, 333, 4097, 20001, 1590], np.int32)
    c2 = np.array([0, 5, 300, 334, 9000, 20002, 2000], np.int32)
    got, full = _partial_ranges(ctx, oracle, q, kp, vp, table, lens,
                                [np.zeros(B, np.int32), c1, c2, lens], H, Hkv, d, bs, "bf16")
    assert np.max(np.abs(got - full)) <= BF16_ATOL


def test_bf16_partial_one_kv_head_long(ctx, oracle):
    """One kv head over 131072-token ranges: every range spreads over hundreds of
    warps, so the partial form's grid-barrier merge runs."""
    rng = np.random.default_rng(22)
    B, H, Hkv, d, bs, L = 2, 8, 1, 128, 16, 131072
    q, kp, vp, table, lens = decode_case(rng, B, [L, L - 9], H, Hkv, d, bs, 2 * L // bs)
    mid = np.array([65536 + 8, 1000], np.int32)
    got, full = _partial_ranges(ctx, oracle, q, kp, vp, table, lens,
                                [np.zeros(B, np.int32), mid, lens], H, Hkv, d, bs, "bf16")
    assert np.max(np.abs(got - full)) <= BF16_ATOL


def test_bf16_c5_long_context(ctx, oracle):
    """Config C5: 64 q / 8 kv heads, 8 sequences x 131072 tokens, 65536-block pool. All heads
    run on the GPU; kv head group 3 (query heads 24-31) of every sequence is checked against
    the oracle (a one-group slice of the pool keeps the host copy at 0.5 GB)."""
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(131072)
    B, H, Hkv, d, bs, nb, L = 8, 64, 8, 128, 16, 65536, 131072
    nblk = L // bs
    perm = rng.permutation(nb).astype(np.int32)
    table = perm.reshape(B, nblk).copy()
    lens = np.full(B, L, np.int32)
    g = torch.Generator(device="cuda").manual_seed(5)
    tk = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    tv = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    tq = torch.randn((B, H, d), generator=g, device="cuda").to(torch.bfloat16)
    out = torch.full_like(tq, float("nan"))
    zb.CudaAttention(ctx).paged_forward(tq, tk, tv, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(),
                                        out, B, H, Hkv, d, bs, nblk, num_blocks=nb)
    ctx.check_status()
    kvh = 3
    k32 = tk[:, kvh:kvh + 1].float().cpu().numpy()
    v32 = tv[:, kvh:kvh + 1].float().cpu().numpy()
    q32 = tq[:, 8 * kvh: 8 * kvh + 8].float().cpu().numpy()
    ref = oracle.paged_decode(q32, k32, v32, table, lens, 8, 1, d, bs, nb, num_threads=8)
    got = out[:, 8 * kvh: 8 * kvh + 8].float().cpu().numpy()
    assert not np.isnan(out.float().cpu().numpy()).any()
    assert np.max(np.abs(got - ref)) <= BF16_ATOL


def test_bf16_one_kv_head_long_split(ctx, oracle):
    """One GPU's shard of C5 at 8 GPUs: a single kv head (8 query heads) over 131072-token
    sequences, so each sequence's stream splits over ~300 warps and the merge combines
    hundreds of partial triples."""
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(77)
    B, H, Hkv, d, bs, L = 2, 8, 1, 128, 16, 131072
    nblk = L // bs
    nb = B * nblk
    table = rng.permutation(nb).astype(np.int32).reshape(B, nblk)
    lens = np.array([L, L - 5], np.int32)
    g = torch.Generator(device="cuda").manual_seed(77)
    tk = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    tv = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    tq = torch.randn((B, H, d), generator=g, device="cuda").to(torch.bfloat16)
    out = torch.full_like(tq, float("nan"))
    zb.CudaAttention(ctx).paged_forward(tq, tk, tv, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(),
                                        out, B, H, Hkv, d, bs, nblk, num_blocks=nb)
    ctx.check_status()
    ref = oracle.paged_decode(tq.float().cpu().numpy(), tk.float().cpu().numpy(), tv.float().cpu().numpy(),
                              table, lens, H, Hkv, d, bs, nb, num_threads=8)
    assert np.max(np.abs(out.float().cpu().numpy() - ref)) <= BF16_ATOL
