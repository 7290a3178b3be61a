"""Varlen prefill on the GPU against the oracle's causal rows (each row is the
CpuAttention last row on its prefix, src/attention/mod.rs:64-97)."""
import numpy as np
import pytest

from helpers import bf16_tensor, f32_tensor, rel_err, to_f32

pytestmark = pytest.mark.gpu


def _case(rng, lens, H, Hkv, d):
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    q = rng.standard_normal((T, H, d)).astype(np.float32)
    k = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    return cu, q, k, v


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("shape", [(4, 4, 8), (8, 2, 64), (4, 1, 128)])
def test_f32_prefill(ctx, oracle, shape, causal):
    import torch
    import zealot_b200 as zb
    H, Hkv, d = shape
    rng = np.random.default_rng(d + H)
    lens = [1, 37, 128, 200]
    cu, q, k, v = _case(rng, lens, H, Hkv, d)
    out = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    zb.CudaAttention(ctx).forward_gpu(f32_tensor(q), f32_tensor(k), f32_tensor(v),
                                      torch.from_numpy(cu).cuda(), out, H, Hkv, d, max(lens),
                                      causal=causal)
    ctx.check_status()
    ref = oracle.prefill_varlen(q, k, v, cu, H, Hkv, d, causal=causal, num_threads=8)
    got = out.cpu().numpy()
    for r in range(q.shape[0]):
        assert rel_err(got[r], ref[r]) <= 1e-4


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("lens", [[1, 127, 128, 129], [300, 700, 5, 1024], [2000]])
def test_bf16_prefill_d128(ctx, oracle, lens, causal):
    """bf16, head_dim 128, GQA 32/8: the tensor-core path (tcgen05) when it applies,
    causal and full (non-causal: every tile of the sequence, the last one masked
    past the sequence end)."""
    import torch
    import zealot_b200 as zb
    H, Hkv, d = 32, 8, 128
    rng = np.random.default_rng(sum(lens))
    cu, q, k, v = _case(rng, lens, H, Hkv, d)
    tq, q32 = bf16_tensor(oracle, q)
    tk, k32 = bf16_tensor(oracle, k)
    tv, v32 = bf16_tensor(oracle, v)
    out = torch.full_like(tq, float("nan"))
    zb.CudaAttention(ctx).forward_gpu(tq, tk, tv, torch.from_numpy(cu).cuda(), out, H, Hkv, d,
                                      max(lens), causal=causal)
    ctx.check_status()
    ref = oracle.prefill_varlen(q32, k32, v32, cu, H, Hkv, d, causal=causal, num_threads=8)
    assert np.max(np.abs(to_f32(out) - ref)) <= 2e-2


def test_bf16_prefill_back_to_back_launches(ctx, oracle):
    """The persistent kernel takes its work items from a device counter that the
    last CTA of each launch returns to zero: launches of different sizes back to
    back on one stream (and one after a launch whose malformed cu_seqlens was
    reported) must each cover all of their items."""
    import torch
    import zealot_b200 as zb
    H, Hkv, d = 32, 8, 128
    attn = zb.CudaAttention(ctx)
    cases = [[1500, 40, 777], [129], [300, 2048, 5, 64, 900]]
    runs = []
    for i, lens in enumerate(cases):
        rng = np.random.default_rng(100 + i)
        cu, q, k, v = _case(rng, lens, H, Hkv, d)
        (tq, q32), (tk, k32), (tv, v32) = (bf16_tensor(oracle, x) for x in (q, k, v))
        runs.append((lens, cu, tq, tk, tv, q32, k32, v32))
    outs = []
    for rep in range(2):
        for lens, cu, tq, tk, tv, *_ in runs:
            out = torch.full_like(tq, float("nan"))
            attn.forward_gpu(tq, tk, tv, torch.from_numpy(cu).cuda(), out, H, Hkv, d, max(lens), causal=True)
            outs.append(out)
        if rep == 0:  # a reported launch in between: sequence 1 ends past total_tokens
            lens, cu, tq, tk, tv, *_ = runs[0]
            bad = cu.copy()
            bad[2] = bad[-1] + 100
            attn.forward_gpu(tq, tk, tv, torch.from_numpy(bad).cuda(), torch.empty_like(tq), H, Hkv, d,
                             max(lens) + 100, causal=True)
            with pytest.raises(zb.OobBlockError):
                ctx.check_status()
    ctx.check_status()
    for r, (lens, cu, tq, tk, tv, q32, k32, v32) in enumerate(runs):
        ref = oracle.prefill_varlen(q32, k32, v32, cu, H, Hkv, d, causal=True, num_threads=8)
        for out in (outs[r], outs[len(runs) + r]):
            assert np.max(np.abs(to_f32(out) - ref)) <= 2e-2


def test_bf16_prefill_c3_sampled(ctx, oracle):
    """Config C3 shape (16 sequences, L U[256, 8192], 32/8 heads, d 128): full GPU run,
    oracle on a seeded sample of rows (first, last, block edges, random)."""
    import torch
    import zealot_b200 as zb
    H, Hkv, d = 32, 8, 128
    rng = np.random.default_rng(3)
    lens = rng.integers(256, 8193, size=16)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    g = torch.Generator(device="cuda").manual_seed(3)
    tq = torch.randn((T, H, d), generator=g, device="cuda").to(torch.bfloat16)
    tk = torch.randn((T, Hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    tv = torch.randn((T, Hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(tq)
    zb.CudaAttention(ctx).forward_gpu(tq, tk, tv, torch.from_numpy(cu).cuda(), out, H, Hkv, d,
                                      int(lens.max()), causal=True)
    ctx.check_status()
    rows = set()
    for s in range(16):
        for i in (0, 1, 127, 128, int(lens[s]) - 1):
            rows.add(int(cu[s]) + min(i, int(lens[s]) - 1))
    rows |= set(int(x) for x in rng.integers(0, T, size=48))
    rows = np.array(sorted(rows), np.int64)
    q32, k32, v32 = (t.float().cpu().numpy() for t in (tq, tk, tv))
    ref = oracle.prefill_varlen_rows(q32, k32, v32, cu, rows, H, Hkv, d, causal=True, num_threads=8)
    got = out.float().cpu().numpy()[rows]
    assert np.max(np.abs(got - ref)) <= 2e-2


def test_bf16_prefill_max_moves_inside_tiles(ctx, oracle):
    """Keys scaled far above the rest sit in the second 64-key half of interior
    tiles (and one in a first half), so for many rows the running max jumps by
    more than 2^8 inside a tile after its first half has already been handed to
    the P V products: the O rescale then waits for those products and the
    second half is taken against the new max. Rows are checked against the oracle."""
    import torch
    import zealot_b200 as zb
    H, Hkv, d = 32, 8, 128
    rng = np.random.default_rng(29)
    lens = [1024, 777]
    cu, q, k, v = _case(rng, lens, H, Hkv, d)
    for pos, factor in ((128 + 100, 12.0), (384 + 70, 25.0), (512 + 10, 30.0), (640 + 127, 40.0),
                        (1024 + 256 + 90, 20.0), (1024 + 512 + 65, 35.0)):
        k[pos] *= factor
    tq, q32 = bf16_tensor(oracle, q)
    tk, k32 = bf16_tensor(oracle, k)
    tv, v32 = bf16_tensor(oracle, v)
    out = torch.full_like(tq, float("nan"))
    zb.CudaAttention(ctx).forward_gpu(tq, tk, tv, torch.from_numpy(cu).cuda(), out, H, Hkv, d,
                                      max(lens), causal=True)
    ctx.check_status()
    ref = oracle.prefill_varlen(q32, k32, v32, cu, H, Hkv, d, causal=True, num_threads=8)
    assert np.max(np.abs(to_f32(out) - ref)) <= 2e-2


def test_bf16_prefill_max_moves_in_first_tile(ctx, oracle):
    """Keys scaled far above the rest in the first key tile of each sequence (both
    64-key halves): every query tile past the diagonal sets its running max from
    them in its first tile, and no later tile comes near it, so the exponentials
    of all later tiles are taken far below the max. Rows are checked against the
    oracle."""
    import torch
    import zealot_b200 as zb
    H, Hkv, d = 32, 8, 128
    rng = np.random.default_rng(31)
    lens = [600, 333]
    cu, q, k, v = _case(rng, lens, H, Hkv, d)
    for pos, factor in ((64 + 36, 30.0), (64 + 63, 20.0), (600 + 5, 15.0), (600 + 64 + 5, 40.0)):
        k[pos] *= factor
    tq, q32 = bf16_tensor(oracle, q)
    tk, k32 = bf16_tensor(oracle, k)
    tv, v32 = bf16_tensor(oracle, v)
    out = torch.full_like(tq, float("nan"))
    zb.CudaAttention(ctx).forward_gpu(tq, tk, tv, torch.from_numpy(cu).cuda(), out, H, Hkv, d,
                                      max(lens), causal=True)
    ctx.check_status()
    ref = oracle.prefill_varlen(q32, k32, v32, cu, H, Hkv, d, causal=True, num_threads=8)
    assert np.max(np.abs(to_f32(out) - ref)) <= 2e-2


@pytest.mark.parametrize("path", ["tcgen05", "generic"])
@pytest.mark.parametrize("bad", ["past_end", "backwards", "longer_than_max"])
def test_malformed_cu_seqlens_is_reported(ctx, oracle, path, bad):
    """cu_seqlens lives in device memory, so the kernels check it: a sequence that
    ends past total_tokens, runs backwards, or is longer than max_seq_len is
    skipped and reported (ZL_ERR_OOB_BLOCK from check_status). `out` is the head of
    a larger buffer whose tail is a guard region: it must come back untouched, and
    the well-formed sequence before the bad one must still match the oracle."""
    import torch
    import zealot_b200 as zb
    H, Hkv, d = (32, 8, 128) if path == "tcgen05" else (4, 2, 64)
    T, guard = 300, 256
    rng = np.random.default_rng(91)
    _, q, k, v = _case(rng, [T], H, Hkv, d)
    good = 120
    cu, max_len = {
        "past_end": (np.array([0, good, T + 40], np.int32), 256),
        "backwards": (np.array([0, good, good - 7], np.int32), 256),
        "longer_than_max": (np.array([0, good, T], np.int32), 128),
    }[bad]
    if path == "tcgen05":
        (tq, q32), (tk, k32), (tv, v32) = (bf16_tensor(oracle, x) for x in (q, k, v))
        dt, tol = torch.bfloat16, 2e-2
    else:
        tq, tk, tv, q32, k32, v32 = f32_tensor(q), f32_tensor(k), f32_tensor(v), q, k, v
        dt, tol = torch.float32, 1e-4
    out_full = torch.full((T + guard, H, d), 7.0, dtype=dt, device="cuda")
    out = out_full[:T]
    zb.CudaAttention(ctx).forward_gpu(tq, tk, tv, torch.from_numpy(cu).cuda(), out, H, Hkv, d, max_len,
                                      causal=True)
    with pytest.raises(zb.OobBlockError):
        ctx.check_status()
    assert torch.all(out_full[T:] == 7.0), "a store left the caller's buffer"
    ref = oracle.prefill_varlen(q32[:good], k32[:good], v32[:good], np.array([0, good], np.int32), H, Hkv, d,
                                causal=True, num_threads=8)
    got = to_f32(out)[:good]
    if path == "tcgen05":
        assert np.max(np.abs(got - ref)) <= tol
    else:
        for r in range(good):
            assert rel_err(got[r], ref[r]) <= tol
