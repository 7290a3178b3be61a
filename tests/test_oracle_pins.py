"""Pins the CPU oracle to the reference's own unit tests (src/attention/mod.rs:117-190,
src/model_runner_cpu.rs:306-401, src/block_manager.rs tests, src/scheduler.rs:601-610)
and checks the restated forms (paged gather, causal rows, partial triples) agree with
the reference CpuAttention they are derived from."""
import numpy as np
import pytest


def test_matmul_known_answer(oracle):
    # attention/mod.rs:183-189
    c = oracle.matmul([1.0, 2.0, 3.0, 4.0], [5.0, 6.0, 7.0, 8.0], 2, 2, 2)
    assert c.tolist() == [19.0, 22.0, 43.0, 50.0]


def test_cpu_attention_single_seq_output_shape(oracle):
    # attention/mod.rs:121-135
    out = oracle.cpu_attention_forward(np.ones(24), np.ones(24), np.ones(24), 1, 2, 4, 3)
    assert out.size == 24


def test_cpu_attention_dimension_mismatch(oracle):
    # attention/mod.rs:137-151
    with pytest.raises(oracle.OracleError):
        oracle.cpu_attention_forward(np.ones(10), np.ones(24), np.ones(24), 1, 2, 4, 3)


def test_cpu_attention_multi_seq_separate(oracle):
    # attention/mod.rs:153-181
    q = np.ones(16, np.float32)
    q[8:] = 100.0
    k = np.array([1, 0, 0, 0, 1, 1, 0, 0, 1, 0, 0, 0, 1, 1, 0, 0], np.float32)
    out = oracle.cpu_attention_forward(q, k, k.copy(), 2, 1, 4, 2)
    assert not np.array_equal(out[:8], out[8:])


def test_repeat_interleave_expands_kv_heads(oracle):
    # model_runner_cpu.rs:323-344
    kv_heads, num_heads, seq_len, d = 2, 4, 3, 2
    src = np.arange(seq_len * kv_heads * d, dtype=np.float32)
    out = oracle.repeat_interleave_kv(src, kv_heads, num_heads, seq_len, d)
    assert out.size == num_heads * seq_len * d
    for head in range(num_heads):
        kh = head % kv_heads
        for pos in range(seq_len):
            for dim in range(d):
                assert out[head * seq_len * d + pos * d + dim] == src[pos * kv_heads * d + kh * d + dim]


def test_repeat_interleave_mha_matches_old_reshape(oracle):
    # model_runner_cpu.rs:346-364
    seq_len, heads, d = 2, 2, 3
    src = np.arange(seq_len * heads * d, dtype=np.float32)
    out = oracle.repeat_interleave_kv(src, heads, heads, seq_len, d)
    expect = np.zeros(heads * seq_len * d, np.float32)
    for head in range(heads):
        for pos in range(seq_len):
            for dim in range(d):
                expect[head * seq_len * d + pos * d + dim] = src[pos * heads * d + head * d + dim]
    assert np.array_equal(out, expect)


def _gqa_fixture_weights():
    # model_runner_cpu.rs:366-382: hidden 8, H 4, Hkv 2, d 2, vocab 4, weights (i % 7) / 7
    rand = lambda n: (np.arange(n) % 7).astype(np.float32) / np.float32(7.0)
    return dict(hidden_dim=8, num_heads=4, num_kv_heads=2, head_dim=2, vocab_size=4,
                embedding=rand(4 * 8), q_proj=rand(8 * 8), k_proj=rand(8 * 4), v_proj=rand(8 * 4),
                attn_proj=rand(8 * 8), lm_head=rand(8 * 4))


def test_gqa_step_no_panic(oracle):
    # model_runner_cpu.rs:366-400 (prompt [1, 2, 3]; logits length 4)
    logits = oracle.runner_step(_gqa_fixture_weights(), [1, 2, 3])
    assert logits.shape == (4,)
    assert np.all(np.isfinite(logits))


def test_gqa_step_golden(oracle):
    """Regression pin of the restated runner on the reference's own fixture
    (tests/golden/make_golden.py wrote the values)."""
    g = np.load(_golden("gqa_step.npz"))
    logits = oracle.runner_step(_gqa_fixture_weights(), [1, 2, 3])
    assert np.array_equal(logits, g["logits"])


def _golden(name):
    import os
    return os.path.join(os.path.dirname(__file__), "golden", name)


def test_argmax_first_max_wins(oracle):
    # sampling.rs:233-243
    assert oracle.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert oracle.argmax([-np.inf, -np.inf]) == 0


def test_block_manager_model_lifo_and_generation(oracle):
    # block_manager.rs:93-95 (ids 0,1,2,...), :102 (generation starts at 1), LIFO reuse
    bm = oracle.OracleBlockManager(4, 16)
    hs = [bm.try_allocate() for _ in range(3)]
    assert [h[0] for h in hs] == [0, 1, 2] and all(h[1] == 1 for h in hs)
    bm.try_free(hs[1])
    h = bm.try_allocate()
    assert h == (1, 2)
    with pytest.raises(LookupError):
        bm.try_free(hs[1])  # stale
    bm.try_allocate()
    with pytest.raises(MemoryError):
        bm.try_allocate()


def test_step_input_recompute(oracle):
    # scheduler.rs:88-101, :601-610 (recompute input = prompt + outputs)
    assert oracle.step_input([1, 2, 3], [7, 8], True, 0, 512) == [1, 2, 3, 7, 8]
    assert oracle.step_input([1, 2, 3], [7, 8], False, 3, 0) == [8]


def _rand_pool(rng, nb, hkv, bs, d):
    return rng.standard_normal((nb, hkv, bs, d)).astype(np.float32)


def test_paged_decode_equals_cpu_attention_last_row(oracle):
    """The paged gather + row math reproduces CpuAttention's last row bit for bit."""
    rng = np.random.default_rng(0)
    H, Hkv, d, bs, nb = 4, 4, 8, 16, 64
    kp, vp = _rand_pool(rng, nb, Hkv, bs, d), _rand_pool(rng, nb, Hkv, bs, d)
    L = 37
    blocks = rng.permutation(nb)[: (L + bs - 1) // bs].astype(np.int32)
    table = np.full((1, 8), -1, np.int32)
    table[0, : blocks.size] = blocks
    q = rng.standard_normal((1, H, d)).astype(np.float32)
    out = oracle.paged_decode(q, kp, vp, table, [L], H, Hkv, d, bs, nb)
    # dense [1][H][L][d] with the query as the last row
    K = np.stack([kp[blocks[p // bs], :, p % bs, :] for p in range(L)], axis=1)  # [Hkv][L][d]
    V = np.stack([vp[blocks[p // bs], :, p % bs, :] for p in range(L)], axis=1)
    Q = np.zeros((H, L, d), np.float32)
    Q[:, -1, :] = q[0]
    ref = oracle.cpu_attention_forward(Q, K, V, 1, H, d, L).reshape(H, L, d)[:, -1, :]
    assert np.array_equal(out[0], ref)


def test_paged_decode_sentinel_stops(oracle):
    """A negative block-table entry ends the sequence (paged_attention.cu:66-67)."""
    rng = np.random.default_rng(1)
    H, Hkv, d, bs, nb = 2, 2, 8, 16, 8
    kp, vp = _rand_pool(rng, nb, Hkv, bs, d), _rand_pool(rng, nb, Hkv, bs, d)
    q = rng.standard_normal((1, H, d)).astype(np.float32)
    t_full = np.array([[3, 5, 1, 2]], np.int32)
    t_cut = np.array([[3, -1, 1, 2]], np.int32)
    a = oracle.paged_decode(q, kp, vp, t_cut, [64], H, Hkv, d, bs, nb)
    b = oracle.paged_decode(q, kp, vp, t_full, [16], H, Hkv, d, bs, nb)
    assert np.array_equal(a, b)


def test_prefill_rows_equal_runner_last_rows(oracle):
    """Causal row i == CpuAttention last row on the prefix [0, i] (recompute form)."""
    rng = np.random.default_rng(2)
    H, Hkv, d = 2, 1, 8
    lens = [5, 9]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = cu[-1]
    q = rng.standard_normal((T, H, d)).astype(np.float32)
    k = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    out = oracle.prefill_varlen(q, k, v, cu, H, Hkv, d, causal=True)
    for s, L in enumerate(lens):
        for i in range(L):
            r = cu[s] + i
            n = i + 1
            Q = np.zeros((H, n, d), np.float32)
            Q[:, -1, :] = q[r]
            Kd = np.repeat(k[cu[s]: cu[s] + n].transpose(1, 0, 2), H // Hkv, axis=0)
            Vd = np.repeat(v[cu[s]: cu[s] + n].transpose(1, 0, 2), H // Hkv, axis=0)
            ref = oracle.cpu_attention_forward(Q, Kd, Vd, 1, H, d, n).reshape(H, n, d)[:, -1, :]
            assert np.array_equal(out[r], ref)


def test_partials_merge_to_full(oracle):
    rng = np.random.default_rng(3)
    H, Hkv, d, bs, nb = 4, 2, 16, 16, 32
    kp, vp = _rand_pool(rng, nb, Hkv, bs, d), _rand_pool(rng, nb, Hkv, bs, d)
    B = 3
    lens = np.array([40, 77, 5], np.int32)
    table = np.stack([rng.permutation(nb)[:8] for _ in range(B)]).astype(np.int32)
    q = rng.standard_normal((B, H, d)).astype(np.float32)
    full = oracle.paged_decode(q, kp, vp, table, lens, H, Hkv, d, bs, nb)
    cut = np.array([17, 40, 0], np.int32)
    m0, l0, o0 = oracle.paged_decode_partial(q, kp, vp, table, np.zeros(B, np.int32), cut, H, Hkv, d, bs, nb)
    m1, l1, o1 = oracle.paged_decode_partial(q, kp, vp, table, cut, lens, H, Hkv, d, bs, nb)
    merged = oracle.merge_partials(np.stack([m0, m1]), np.stack([l0, l1]), np.stack([o0, o1]))
    np.testing.assert_allclose(merged.reshape(B, H, d), full, rtol=1e-5, atol=1e-6)


def test_store_kv_layout(oracle):
    """kv_cache.rs:245-247 offsets, and slot-mapping form == block-id form."""
    rng = np.random.default_rng(4)
    Hkv, d, bs, nb = 2, 4, 4, 6
    T = 9
    k = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    v = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    block_ids = np.array([4, 1, 3], np.int64)
    kp1, vp1 = np.zeros((nb, Hkv, bs, d), np.float32), np.zeros((nb, Hkv, bs, d), np.float32)
    oracle.store_kv(kp1, vp1, k, v, block_ids, 2, T, Hkv, d, bs)
    for t in range(T):
        p = 2 + t
        assert np.array_equal(kp1[block_ids[p // bs], :, p % bs, :], k[t])
    slots = np.array([block_ids[(2 + t) // bs] * bs + (2 + t) % bs for t in range(T)], np.int64)
    kp2, vp2 = np.zeros_like(kp1), np.zeros_like(vp1)
    assert oracle.reshape_and_cache(kp2, vp2, k, v, slots, Hkv, d, bs, nb) == 0
    assert np.array_equal(kp1, kp2) and np.array_equal(vp1, vp2)
    with pytest.raises(oracle.OracleError):
        oracle.store_kv(kp1, vp1, k, v, block_ids[:1], 0, T, Hkv, d, bs)


def test_bf16_round_trip(oracle):
    x = np.array([1.0, 1.00390625, 1.005859375, -3.14159, 0.0], np.float32)
    b = oracle.f32_to_bf16_bits(x)
    assert b.tolist()[:2] == [0x3F80, 0x3F80]  # ties to even
    assert oracle.bf16_bits_to_f32(b)[2] == np.float32(1.0078125)


# ---- Sampler (src/sampling.rs:292-659): the reference's tests, run on the
# restated sampler with many draws r in place of StdRng::seed_from_u64(42).

_RS = [0.001, 0.01, 0.25, 0.5, 0.75, 0.99, 0.999999]


def _lin(n):
    return np.arange(n, dtype=np.float32)


def test_sampler_temperature_zero_is_greedy(oracle):
    for r in _RS:
        rc, tok, lp, _ = oracle.sample([1.0, 2.0, 3.0, 0.5, 100.0], temperature=0.0, r=r)
        assert rc == 0 and tok == 4 and lp <= 0.0


def test_sampler_temperature_clamp_to_greedy(oracle):
    rc, tok, _, _ = oracle.sample([1.0, 2.0, 50.0, 0.5], temperature=1e-10)
    assert rc == 0 and tok == 2


def test_sampler_greedy_logprob_is_valid(oracle):
    x = np.arange(100, dtype=np.float32) * np.float32(0.1)
    rc, tok, lp, _ = oracle.sample(x, temperature=0.0)
    assert rc == 0 and lp <= 0.0 and lp >= np.log(np.float32(1.0 / 100))


def test_sampler_temperature_scaling_and_top_k_disabled(oracle):
    for r in _RS:
        assert oracle.sample(_lin(10), temperature=100.0, r=r)[1] < 10
        assert oracle.sample(_lin(10), top_k=0, r=r)[1] < 10
        assert oracle.sample(_lin(10), top_p=1.0, r=r)[1] < 10


def test_sampler_top_k(oracle):
    for r in _RS:
        assert oracle.sample([0.1, 5.0, 0.2, 3.0], top_k=1, r=r)[1] == 1
        assert oracle.sample(_lin(100), top_k=3, r=r)[1] >= 97


def test_sampler_penalties(oracle):
    for r in _RS:
        assert oracle.sample([1.0, 2.0, 100.0, 0.5], prev=[2, 2], r=r)[1] == 2
        # p = [0.00055, 0.0300, 0.603, 0.366]: token 2 for 0.0306 <= r < 0.634
        if 0.04 < r < 0.6:
            assert oracle.sample([1.0, 5.0, 8.0, 7.5], prev=[1], r=r)[1] == 2
            assert oracle.sample([1.0, 5.0, 8.0, 7.5], prev=[1], repetition_penalty=1.5, r=r)[1] == 2
        assert oracle.sample([1.0, 100.0, 1.0, 1.0], prev=[1] * 8, frequency_penalty=30.0, r=r)[1] != 1
        assert oracle.sample([10.0, 15.0, 5.0, 12.0], prev=[1], presence_penalty=10.0, r=r)[1] != 1
    # penalty arithmetic itself: 5.0 / 1.5 for a positive logit, x * 1.5 for a negative one,
    # once per occurrence; greedy ignores penalties (the fast path comes first)
    rc, tok, _, _ = oracle.sample([1.0, 5.0, 8.0, 7.5], prev=[1], repetition_penalty=1.5, top_k=1)
    assert (rc, tok) == (0, 2)
    assert oracle.sample([3.0, 2.9], prev=[0, 0], repetition_penalty=1.1, top_k=1)[1] == 1
    assert oracle.sample([3.0, 2.9], prev=[0, 0], repetition_penalty=1.1, temperature=0.0)[1] == 0


def test_sampler_errors(oracle):
    assert oracle.sample([])[0] == oracle.EMPTY_LOGITS
    assert oracle.sample([-np.inf] * 10)[0] == oracle.ALL_TOKENS_MASKED
    assert oracle.sample([1.0, 2.0, 3.0], mask=[0, 0, 0])[0] == oracle.ALL_TOKENS_MASKED


def test_sampler_masks(oracle):
    assert oracle.sample([1.0, 5.0, 3.0, 4.0], mask=[0, 0, 1, 0], temperature=0.0)[1] == 2
    assert oracle.sample([1.0, 100.0, 2.0, 3.0], mask=[1, 0, 1, 1], top_k=1)[1] == 3
    assert oracle.sample([1.0, 2.0, 3.0, 4.0, 5.0], mask=[0, 0, 1], temperature=0.0)[1] == 4
    assert (oracle.sample([1.0, 2.0, 100.0], temperature=0.0)[1]
            == oracle.sample([1.0, 2.0, 100.0], temperature=0.0, mask=None)[1])


def test_sampler_deterministic_and_combined(oracle):
    a = oracle.sample(_lin(50), temperature=0.8, top_k=10, r=0.3)
    b = oracle.sample(_lin(50), temperature=0.8, top_k=10, r=0.3)
    assert a[1] == b[1] and abs(a[2] - b[2]) < 1e-6
    for r in _RS:
        rc, tok, lp, _ = oracle.sample(_lin(100), prev=[99, 98, 97], temperature=0.7, top_k=20,
                                       top_p=0.9, repetition_penalty=1.2, frequency_penalty=0.5,
                                       presence_penalty=0.3, r=r)
        assert rc == 0 and tok < 100 and lp <= 0.0
        assert tok >= 80  # top-k 20 keeps 80..99


def test_sampler_multinomial_cdf(oracle):
    """sample_multinomial (sampling.rs:276-290): the first i with r < cdf(i)."""
    x = np.log(np.array([0.1, 0.2, 0.3, 0.4], np.float32))
    assert [oracle.sample(x, r=r)[1] for r in (0.05, 0.15, 0.35, 0.65, 0.95)] == [0, 1, 2, 3, 3]


def test_sampler_softmax(oracle):
    """softmax_sums_to_one and softmax_stable_with_extreme_values (sampling.rs:620-645)."""
    p = oracle.softmax([1.0, 2.0, 3.0, 4.0, 5.0])
    assert abs(float(np.sum(p, dtype=np.float32)) - 1.0) < 1e-5
    p = oracle.softmax([1e5, -1e5, 0.0, 5e4])
    assert abs(float(np.sum(p, dtype=np.float32)) - 1.0) < 1e-5 and np.isfinite(p).all()
