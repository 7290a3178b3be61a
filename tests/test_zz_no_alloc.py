"""The allocation-free paged decode (zl_paged_decode_noalloc), called through
the C ABI.

Some callers of this library cannot allocate device memory while they serve:
an engine that gives nearly all of its HBM to the KV-cache pool at start-up
has nothing left for the split-KV workspace zl_paged_decode grows with
cudaMalloc, and a step loop that must not stall cannot take the device-wide
synchronisation cudaMalloc implies. The allocation-free entry point keeps
that scratch in a static device array instead.

Both entry points run the same kernel over the same grid, so the same inputs
split the same way and merge in the same order: their outputs must be equal
byte for byte. The GPU tests check that on two calls in a row with different
batches (long contexts, so sequences split across warps and the scratch is
really used), at the largest batch the scratch admits, and against the CPU
oracle on a small case (2e-2 absolute, the bf16 tolerance of the other decode
tests); they also check that a bad block id reaches the caller's status word.
The size and argument checks return before any CUDA call and run on the CPU.

The file name sorts last so that, in a run that stops at the first failure,
every other test has already run.
"""
import numpy as np
import pytest

BF16_ATOL = 2e-2
MAX_SEQS, MAX_PAIRS = 4096, 16384


def _batch(seed, B, H, d, bs, nb, lo=1, hi=16000):
    import torch
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi, size=B).astype(np.int32)
    lens[0] = 0                        # an empty context
    if B > 1:
        lens[1] = 16 * 37              # an exact multiple of the block size
    nblk = (lens + bs - 1) // bs
    mb = int(nblk.max())
    perm = rng.permutation(nb).astype(np.int32)
    table = np.full((B, mb), -1, np.int32)
    off = 0
    for b in range(B):
        table[b, : nblk[b]] = perm[off: off + nblk[b]]
        off += nblk[b]
    assert off <= nb
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn((B, H, d), generator=g, device="cuda").to(torch.bfloat16)
    return q, table, lens, mb


def _pools(seed, nb, Hkv, bs, d):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    vp = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    return kp, vp


def _noalloc(q, kp, vp, table, lens, out, status, H, Hkv, d, bs, mb, nb):
    import torch
    import zealot_b200 as zb
    from zealot_b200.context import ptr
    B = q.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    rc = zb.lib.zl_paged_decode_noalloc(ptr(q), ptr(kp), ptr(vp), ptr(table), ptr(lens), ptr(out), ptr(status),
                                        B, H, Hkv, d, bs, mb, nb, 0.0, stream)
    assert rc == 0, zb.lib.zl_last_error()


def _with_context(ctx, q, kp, vp, table, lens, H, Hkv, d, bs, mb, nb):
    import torch
    import zealot_b200 as zb
    ref = torch.full_like(q, float("nan"))
    zb.CudaAttention(ctx).paged_forward(q, kp, vp, table, lens, ref, q.shape[0], H, Hkv, d, bs, mb,
                                        num_blocks=nb)
    ctx.check_status()
    return ref


@pytest.mark.gpu
def test_noalloc_equals_paged_decode_twice(ctx):
    import torch
    B, H, Hkv, d, bs, nb = 24, 32, 8, 128, 16, 16384
    kp, vp = _pools(77, nb, Hkv, bs, d)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call, seed in enumerate((1, 2)):
        q, table, lens, mb = _batch(seed, B, H, d, bs, nb)
        tt, tl = torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda()
        ref = _with_context(ctx, q, kp, vp, tt, tl, H, Hkv, d, bs, mb, nb)
        out = torch.full_like(q, float("nan"))
        _noalloc(q, kp, vp, tt, tl, out, status, H, Hkv, d, bs, mb, nb)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.all(out[0].float() == 0)      # empty context writes zeros
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {call}: bytes differ"


@pytest.mark.gpu
def test_noalloc_small_case_against_oracle(oracle):
    import torch
    from helpers import bf16_tensor, decode_case
    rng = np.random.default_rng(31)
    B, H, Hkv, d, bs, nb = 5, 16, 2, 128, 16, 512
    q, kp, vp, table, lens = decode_case(rng, B, [0, 1, 17, 700, 2500], H, Hkv, d, bs, nb)
    (tq, q32), (tk, k32), (tv, v32) = (bf16_tensor(oracle, x) for x in (q, kp, vp))
    out = torch.full_like(tq, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _noalloc(tq, tk, tv, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), out, status,
             H, Hkv, d, bs, table.shape[1], nb)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = oracle.paged_decode(q32, k32, v32, table, lens, H, Hkv, d, bs, nb, num_threads=8)
    assert np.max(np.abs(out.float().cpu().numpy() - ref)) <= BF16_ATOL


@pytest.mark.gpu
def test_noalloc_at_the_segment_limit(ctx):
    """2048 sequences x 8 kv heads = 16384 (sequence, kv head) pairs, the most the
    static scratch admits: every merge counter of the array is in use."""
    import torch
    B, H, Hkv, d, bs, nb = 2048, 32, 8, 128, 16, 16384
    assert B * Hkv == MAX_PAIRS
    kp, vp = _pools(78, nb, Hkv, bs, d)
    q, table, lens, mb = _batch(5, B, H, d, bs, nb, lo=1, hi=100)
    tt, tl = torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda()
    ref = _with_context(ctx, q, kp, vp, tt, tl, H, Hkv, d, bs, mb, nb)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _noalloc(q, kp, vp, tt, tl, out, status, H, Hkv, d, bs, mb, nb)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.gpu
def test_noalloc_reports_a_block_outside_the_pool():
    """A block id >= num_blocks is skipped by the kernel's bounds check and flagged
    in the caller's status word (bit 0); the call itself returns ZL_OK."""
    import torch
    B, H, Hkv, d, bs, nb = 2, 8, 2, 128, 16, 64
    kp, vp = _pools(79, nb, Hkv, bs, d)
    q, table, lens, mb = _batch(6, B, H, d, bs, nb, lo=40, hi=200)
    table[1, 1] = nb + 5
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    _noalloc(q, kp, vp, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), out, status,
             H, Hkv, d, bs, mb, nb)
    torch.cuda.synchronize()
    assert int(status.item()) & 1


def _reject(B, H, Hkv, status_ptr=16):
    import zealot_b200 as zb
    rc = zb.lib.zl_paged_decode_noalloc(16, 16, 16, 16, 16, 16, status_ptr, B, H, Hkv, 128, 16, 4, 64, 0.0,
                                        None)
    return rc, zb.lib.zl_last_error()


def test_noalloc_rejects_too_many_sequences():
    import zealot_b200 as zb
    rc, msg = _reject(MAX_SEQS + 1, 32, 8)
    assert rc == zb.InvalidArgument.status and b"static scratch" in msg


def test_noalloc_rejects_too_many_pairs():
    """3277 sequences x 5 kv heads = 16385 pairs: one past the scratch's counters."""
    import zealot_b200 as zb
    assert 3277 * 5 == MAX_PAIRS + 1
    rc, msg = _reject(3277, 5, 5)
    assert rc == zb.InvalidArgument.status and b"static scratch" in msg


def test_noalloc_requires_a_status_word():
    import zealot_b200 as zb
    rc, msg = _reject(4, 32, 8, status_ptr=None)
    assert rc == zb.InvalidArgument.status and b"status word" in msg
