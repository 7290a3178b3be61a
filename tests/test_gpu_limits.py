"""Argument limits of the attention entry points, called through the C ABI.

- Invalid arguments come back as ZL_ERR_INVALID_ARG (InvalidArgument) and head
  dims past 256 as ZL_ERR_UNSUPPORTED, before any kernel is launched, like the
  reference's Result::Err(ZealotError) on bad input (src/attention/mod.rs:121-181
  shape tests); the context stays usable.
- Zero-sized batches are no-ops, whatever the pointers (the engine calls the
  runner with empty decode or prefill sets, src/engine.rs:145-228).
- bf16 shapes outside the tensor-core / fast paths (odd GQA group, head_dim 64,
  more than 8 query heads per kv head) fall back to the generic kernels and
  still match the oracle within the bf16 tolerance (2e-2 absolute).
- A device wait that nothing satisfies ends on its own budget and is reported as
  DeviceTimeout (failure detection without a GPU fault).
"""
import numpy as np
import pytest

from helpers import bf16_tensor, decode_case, to_f32

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2


def _raw(ctx):
    import torch
    from zealot_b200.context import dtype_code, ptr
    bufs = {
        "bf16": torch.zeros(1 << 16, dtype=torch.bfloat16, device="cuda"),
        "i32": torch.zeros(64, dtype=torch.int32, device="cuda"),
        "i64": torch.zeros(64, dtype=torch.int64, device="cuda"),
        "f32": torch.zeros(1 << 16, dtype=torch.float32, device="cuda"),
    }
    p = {k: ptr(v) for k, v in bufs.items()}
    return ctx.lib, ctx.handle, torch.cuda.current_stream().cuda_stream, dtype_code(torch.bfloat16), p, bufs


def test_entry_points_reject_bad_arguments(ctx, oracle):
    import zealot_b200 as zb
    from zealot_b200.errors import check
    lib, h, st, BF, p, _keep = _raw(ctx)
    b, i32, i64, f32 = p["bf16"], p["i32"], p["i64"], p["f32"]

    def dec(q=b, B=2, H=4, Hkv=2, d=128, bs=16, mb=4, nb=8, dt=BF):
        return lib.zl_paged_decode(h, q, b, b, i32, i32, b, B, H, Hkv, d, bs, mb, nb, 0.0, 0, 0, dt, st)

    def pre(q=b, n=1, maxl=8, T=8, H=4, Hkv=2, d=128, dt=BF):
        return lib.zl_prefill_varlen(h, q, b, b, i32, n, maxl, T, b, H, Hkv, d, 0.0, 1, 0, dt, st)

    def cache(k=b, T=2, Hkv=2, d=128, bs=16, nb=4, dt=BF):
        return lib.zl_reshape_and_cache(h, k, b, b, b, i64, T, Hkv, d, bs, nb, dt, st)

    def merge(P=2, rows=4, d=128, dt=BF):
        return lib.zl_merge_partials(h, f32, f32, f32, P, rows, d, b, dt, st)

    bad = ([(dec, kw) for kw in (dict(H=5), dict(Hkv=0), dict(d=0), dict(bs=0), dict(B=-1), dict(mb=-1),
                                 dict(nb=-1), dict(q=None), dict(dt=99))]
           + [(pre, kw) for kw in (dict(H=3), dict(Hkv=0), dict(n=-1), dict(maxl=-1), dict(T=-1),
                                   dict(q=None), dict(dt=99))]
           + [(cache, kw) for kw in (dict(T=-1), dict(Hkv=0), dict(d=0), dict(bs=0), dict(nb=-1),
                                     dict(k=None), dict(dt=99))]
           + [(merge, kw) for kw in (dict(P=0), dict(rows=-1), dict(d=0), dict(dt=99))])
    for fn, kw in bad:
        with pytest.raises(zb.InvalidArgument):
            check(fn(**kw))
    # head dims past the kernels' limit (256) are refused, not launched
    for fn in (dec, pre):
        with pytest.raises(zb.Unsupported):
            check(fn(d=512))
    ctx.check_status()  # nothing ran, nothing was flagged
    # the context still works: a small decode against the oracle
    rng = np.random.default_rng(11)
    H, Hkv, d, bs = 8, 2, 128, 16
    q, kp, vp, table, lens = decode_case(rng, 3, [5, 40, 300], H, Hkv, d, bs, 64)
    got, ref = _decode_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs)
    assert np.max(np.abs(got - ref)) <= BF16_ATOL


def test_zero_sized_calls_are_noops(ctx):
    from zealot_b200.errors import check
    lib, h, st, BF, p, _keep = _raw(ctx)
    # every pointer null: an empty batch must not touch them
    check(lib.zl_paged_decode(h, None, None, None, None, None, None, 0, 32, 8, 128, 16, 4, 8, 0.0, 0, 0,
                              BF, st))
    check(lib.zl_prefill_varlen(h, None, None, None, None, 0, 0, 0, None, 32, 8, 128, 0.0, 1, 0, BF, st))
    check(lib.zl_prefill_varlen(h, None, None, None, None, 4, 64, 0, None, 32, 8, 128, 0.0, 1, 0, BF, st))
    check(lib.zl_reshape_and_cache(h, None, None, None, None, None, 0, 8, 128, 16, 4, BF, st))
    check(lib.zl_merge_partials(h, None, None, None, 2, 0, 128, None, BF, st))
    ctx.check_status()


def _decode_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs):
    import torch
    import zealot_b200 as zb
    tq, q32 = bf16_tensor(oracle, q)
    tk, k32 = bf16_tensor(oracle, kp)
    tv, v32 = bf16_tensor(oracle, vp)
    out = torch.full_like(tq, float("nan"))
    zb.CudaAttention(ctx).paged_forward(tq, tk, tv, torch.from_numpy(table).cuda(),
                                        torch.from_numpy(np.asarray(lens, np.int32)).cuda(), out,
                                        table.shape[0], H, Hkv, d, bs, table.shape[1],
                                        num_blocks=kp.shape[0])
    ctx.check_status()
    ref = oracle.paged_decode(q32, k32, v32, table, lens, H, Hkv, d, bs, kp.shape[0], num_threads=8)
    return to_f32(out), ref


@pytest.mark.parametrize("H,Hkv,d", [(32, 2, 128), (8, 2, 64), (6, 2, 128)])
def test_bf16_decode_outside_fast_path(ctx, oracle, H, Hkv, d):
    """16 query heads per kv head, head_dim 64, a group of 3: the generic kernel."""
    rng = np.random.default_rng(H * 100 + d)
    q, kp, vp, table, lens = decode_case(rng, 4, [1, 17, 160, 999], H, Hkv, d, 16, 128)
    got, ref = _decode_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, 16)
    assert np.max(np.abs(got - ref)) <= BF16_ATOL


@pytest.mark.parametrize("H,Hkv,d", [(6, 2, 128), (8, 2, 64), (3, 3, 128)])
def test_bf16_prefill_outside_tensor_core_path(ctx, oracle, H, Hkv, d):
    """An odd GQA group (3), head_dim 64 and MHA with an odd head count: the
    generic kernel; causal rows against the oracle's prefix rows."""
    import torch
    import zealot_b200 as zb
    rng = np.random.default_rng(H * 10 + d)
    lens = [1, 130, 257]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    q = rng.standard_normal((T, H, d)).astype(np.float32)
    k = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    tq, q32 = bf16_tensor(oracle, q)
    tk, k32 = bf16_tensor(oracle, k)
    tv, v32 = bf16_tensor(oracle, v)
    out = torch.full_like(tq, float("nan"))
    zb.CudaAttention(ctx).forward_gpu(tq, tk, tv, torch.from_numpy(cu).cuda(), out, H, Hkv, d, max(lens),
                                      causal=True)
    ctx.check_status()
    ref = oracle.prefill_varlen(q32, k32, v32, cu, H, Hkv, d, causal=True, num_threads=8)
    assert np.max(np.abs(to_f32(out) - ref)) <= BF16_ATOL


def test_bounded_wait_times_out_and_context_recovers(ctx, oracle):
    """A device wait that nothing satisfies gives up on its own budget (about a
    second), flags the status word (DeviceTimeout on the host) and leaves the
    context usable: no trap, no hang."""
    import time
    import zealot_b200 as zb
    from zealot_b200.errors import check
    ctx.check_status()
    t0 = time.perf_counter()
    check(ctx.lib.zl_selftest_wait_timeout(ctx.handle, ctx.stream()))
    with pytest.raises(zb.DeviceTimeout):
        ctx.check_status()
    assert 0.05 < time.perf_counter() - t0 < 60
    ctx.check_status()  # the word was cleared by the first read
    rng = np.random.default_rng(12)
    H, Hkv, d, bs = 8, 2, 128, 16
    q, kp, vp, table, lens = decode_case(rng, 3, [7, 99, 700], H, Hkv, d, bs, 64)
    got, ref = _decode_bf16(ctx, oracle, q, kp, vp, table, lens, H, Hkv, d, bs)
    assert np.max(np.abs(got - ref)) <= BF16_ATOL
