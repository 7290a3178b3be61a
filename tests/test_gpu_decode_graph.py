"""Device-resident decode loop (zl_decode_graph_*).

1. Against a host-managed loop built from the same parts (StepBatch.build ->
   zl_decoder_step -> zl_sample with host penalty lists, blocks allocated on the
   host): identical tokens, logprobs and pool bytes after 40 steps that cross
   block boundaries, with greedy, top-k, top-p and penalty rows. At four of the
   steps the graph's logits are also checked against the plain PyTorch fp32
   restatement of the layer loop (test_gpu_decoder.reference_step) run on fp32
   copies of the same pools, within the decoder test's tolerance, so the
   replayed steps are tied to an independent reference, not only to the same
   kernels issued from the host.
2. The captured graph against the same launches issued eagerly, with an
   inactive row and a row recycled mid-run: identical tokens.
3. Host-side errors: a missing or unexpected block.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BS = 16
MAXB = 16


def _setup(ctx, seed=3, with_weights=False):
    from test_gpu_decoder import _cfg
    from zealot_b200.decoder import Decoder, random_weights
    cfg = _cfg(layers=2)
    w = random_weights(cfg, seed=seed)
    dec = Decoder(ctx, cfg, w)
    return (cfg, dec, w) if with_weights else (cfg, dec)


def _prefill(dec, prompts, tables, pools):
    from zealot_b200.decoder import StepBatch
    batch = StepBatch.build(prompts, [], None, [], tables, BS)
    return dec.step(batch, pools[0], pools[1], BS)


def _params():
    from zealot_b200.sampling import SamplingParams as SP
    return [SP(temperature=0.0), SP(temperature=0.8, top_k=40), SP(top_p=0.9, repetition_penalty=1.3),
            SP(temperature=1.1, frequency_penalty=0.4, presence_penalty=0.2)]


def test_decode_graph_matches_host_loop(ctx):
    import torch
    from zealot_b200.decoder import DecodeGraph, StepBatch
    from zealot_b200.sampling import GpuSampler
    from test_gpu_decoder import reference_step
    cfg, dec, w = _setup(ctx, with_weights=True)
    rng = np.random.default_rng(0)
    lens0 = [30, 47, 16, 5]
    prompts = [rng.integers(0, cfg.vocab, n) for n in lens0]
    free = list(rng.permutation(256))
    tables = [[int(free.pop()) for _ in range((n + BS - 1) // BS)] for n in lens0]
    pools_a = dec.new_pools(256, BS)
    logits = _prefill(dec, prompts, tables, pools_a)
    pools_b = ([t.clone() for t in pools_a[0]], [t.clone() for t in pools_a[1]])
    params = _params()
    sampler = GpuSampler(ctx)
    u0 = rng.random(4).astype(np.float32)
    first = sampler.sample(logits, params, None, None, u0).token_ids.cpu().numpy()
    free_b = list(free)

    # host-managed loop
    toks, lens, hist = first.copy(), list(lens0), [[int(t)] for t in first]
    tabs_a = [list(t) for t in tables]
    draws = rng.random((40, 4)).astype(np.float32)
    want_tok, want_lp = [], []
    for t in range(40):
        for r in range(4):
            if lens[r] % BS == 0:
                tabs_a[r].append(int(free.pop()))
        lens = [n + 1 for n in lens]
        dt = np.full((4, MAXB), -1, np.int32)
        for r in range(4):
            dt[r, : len(tabs_a[r])] = tabs_a[r]
        batch = StepBatch.build([], toks, dt, lens, [], BS)
        lg = dec.step(batch, pools_a[0], pools_a[1], BS)
        out = sampler.sample(lg, params, hist, None, draws[t])
        toks = out.token_ids.cpu().numpy()
        want_tok.append(toks.copy())
        want_lp.append(out.logprobs.cpu().numpy())
        for r in range(4):
            hist[r].append(int(toks[r]))
    ctx.check_status()

    g = DecodeGraph(dec, pools_b[0], pools_b[1], BS, rows=4, max_blocks_per_seq=MAXB)
    assert g.num_kernels > 4 * cfg.num_layers
    for r in range(4):
        g.set_row(r, tables[r], lens0[r], int(first[r]), params[r], history=[int(first[r])])
    tabs_b, lens_b, toks_b = [list(t) for t in tables], list(lens0), first.copy()
    checked = 0
    for t in range(40):
        need = g.rows_needing_block()
        new = {r: int(free_b.pop()) for r in need}
        for r, blk in new.items():
            tabs_b[r].append(blk)
        lens_b = [n + 1 for n in lens_b]
        anchor = t in (0, 15, 16, 39)
        if anchor:  # fp32 copies of the pools as this step finds them
            k32 = [p.float() for p in pools_b[0]]
            v32 = [p.float() for p in pools_b[1]]
        g.step(new, draws[t])
        tok, lp = g.tokens()
        assert (tok == want_tok[t]).all(), (t, tok, want_tok[t])
        np.testing.assert_array_equal(lp, want_lp[t])
        if anchor:
            dt = np.full((4, MAXB), -1, np.int32)
            for r in range(4):
                dt[r, : len(tabs_b[r])] = tabs_b[r]
            ref = reference_step(cfg, w, StepBatch.build([], toks_b, dt, lens_b, [], BS), k32, v32,
                                 round_bf16=True)
            torch.testing.assert_close(torch.from_numpy(g.logits()), ref.cpu(), atol=2e-2, rtol=2e-2)
            checked += 1
        toks_b = tok
    assert checked == 4
    ctx.check_status()
    for l in range(cfg.num_layers):
        assert torch.equal(pools_a[0][l], pools_b[0][l]) and torch.equal(pools_a[1][l], pools_b[1][l])
    g.close()


def test_decode_graph_replay_equals_eager_with_recycled_rows(ctx):
    from zealot_b200.decoder import DecodeGraph
    from zealot_b200.sampling import GpuSampler
    cfg, dec = _setup(ctx, seed=8)
    rng = np.random.default_rng(1)
    lens0 = [21, 64, 9]
    prompts = [rng.integers(0, cfg.vocab, n) for n in lens0]
    new_prompt = rng.integers(0, cfg.vocab, 40)
    perm = list(rng.permutation(256))
    tables = [[int(perm.pop()) for _ in range((n + BS - 1) // BS)] for n in lens0]
    new_table = [int(perm.pop()) for _ in range(3)]
    params = _params()
    draws = rng.random((24, 4)).astype(np.float32)
    runs = []
    for use_graph in (True, False):
        pools = dec.new_pools(256, BS)
        logits = _prefill(dec, prompts, tables, pools)
        first = GpuSampler(ctx).sample(logits, params[:3], None, None, draws[0][:3]).token_ids.cpu().numpy()
        g = DecodeGraph(dec, pools[0], pools[1], BS, rows=4, max_blocks_per_seq=MAXB, use_graph=use_graph)
        for r in range(3):  # row 3 stays inactive
            g.set_row(r, tables[r], lens0[r], int(first[r]), params[r], history=[int(first[r])])
        free = list(perm)
        out = []
        for t in range(24):
            if t == 12:  # row 1 finishes; a new sequence takes it after its prefill
                g.clear_row(1)
                lg = _prefill(dec, [new_prompt], [new_table], pools)
                nt = int(lg[0].argmax())
                g.set_row(1, new_table, 40, nt, params[0], history=[nt])
            g.step({r: int(free.pop()) for r in g.rows_needing_block()}, draws[t])
            out.append(g.tokens()[0][:3].copy())
        ctx.check_status()
        g.close()
        runs.append(np.stack(out))
    np.testing.assert_array_equal(runs[0], runs[1])


def test_decode_graph_host_errors(ctx):
    import zealot_b200 as zb
    from zealot_b200.decoder import DecodeGraph
    cfg, dec = _setup(ctx)
    pools = dec.new_pools(64, BS)
    g = DecodeGraph(dec, pools[0], pools[1], BS, rows=2, max_blocks_per_seq=4, use_graph=False)
    g.set_row(0, [3], 16, 5)  # the next token opens a second block
    assert g.rows_needing_block() == [0]
    u = np.zeros(2, np.float32)
    with pytest.raises(zb.InvalidArgument):
        g.step({}, u)                # the block is missing
    with pytest.raises(zb.InvalidArgument):
        g.step({0: 7, 1: 8}, u)      # row 1 needs none
    with pytest.raises(zb.InvalidArgument):
        g.step({0: 64}, u)           # outside the pool
    with pytest.raises(zb.InvalidArgument):
        g.set_row(1, [99], 4, 1)     # block id outside the pool
    g.step({0: 7}, u)
    assert g.rows_needing_block() == []
    ctx.check_status()
    g.set_row(1, [1, 2, 4, 5], 64, 1)
    with pytest.raises(zb.SequenceTooLong):
        g.rows_needing_block()
    g.close()
