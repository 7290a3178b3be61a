"""The allocation-free paged decode (zl_paged_decode_noalloc), called through
the C ABI, against the context-based zl_paged_decode.

Some callers of this library cannot allocate device memory while they serve:
an engine that gives nearly all of its HBM to the KV-cache pool at start-up
has nothing left for the split-KV workspace zl_paged_decode grows with
cudaMalloc, and a step loop that must not stall cannot take the device-wide
synchronisation cudaMalloc implies. The allocation-free entry point keeps
that scratch in a static device array instead. This test runs it twice in a
row on different batches (long contexts, so sequences split across warps and
the scratch is really used) and checks each output against zl_paged_decode
within the bf16 tolerance of the other decode tests (2e-2 absolute).

The file name sorts last so that, in a run that stops at the first failure,
every other test has already run.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2


def _batch(seed, B, H, Hkv, d, bs, nb):
    import torch
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 16000, size=B).astype(np.int32)
    lens[0] = 0                        # an empty context
    lens[1] = 16 * 37                  # an exact multiple of the block size
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
    return q, torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), mb


def test_noalloc_matches_paged_decode_twice(ctx):
    import torch
    import zealot_b200 as zb
    from zealot_b200.context import ptr
    lib = zb.lib
    B, H, Hkv, d, bs, nb = 24, 32, 8, 128, 16, 16384
    g = torch.Generator(device="cuda").manual_seed(77)
    kp = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    vp = torch.randn((nb, Hkv, bs, d), generator=g, device="cuda").to(torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for call, seed in enumerate((1, 2)):
        q, table, lens, mb = _batch(seed, B, H, Hkv, d, bs, nb)
        ref = torch.full_like(q, float("nan"))
        zb.CudaAttention(ctx).paged_forward(q, kp, vp, table, lens, ref, B, H, Hkv, d, bs, mb,
                                            num_blocks=nb)
        ctx.check_status()
        out = torch.full_like(q, float("nan"))
        st_ptr = 0 if call == 0 else ptr(status)   # first call: no status word
        rc = lib.zl_paged_decode_noalloc(ptr(q), ptr(kp), ptr(vp), ptr(table), ptr(lens), ptr(out),
                                         st_ptr, B, H, Hkv, d, bs, mb, nb, 0.0, stream)
        assert rc == 0, lib.zl_last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert not torch.isnan(out.float()).any()
        assert torch.all(out[0].float() == 0)      # empty context writes zeros
        diff = (out.float() - ref.float()).abs().max().item()
        assert diff <= BF16_ATOL, f"call {call}: max abs diff {diff}"


def test_noalloc_rejects_oversized_batch():
    import zealot_b200 as zb
    lib = zb.lib
    # 4097 sequences: beyond the static scratch limit; rejected before any launch
    rc = lib.zl_paged_decode_noalloc(16, 16, 16, 16, 16, 16, 0, 4097, 32, 8, 128, 16, 4, 64, 0.0, None)
    assert rc == zb.InvalidArgument.status
    assert b"static scratch" in lib.zl_last_error()
