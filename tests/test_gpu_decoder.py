"""Full-decoder engine step (the layer loop of src/cuda_runner.rs:303-607, batched)
against a plain PyTorch fp32 reference of the same model.

Two references:
* `bf16-matched`: fp32 math that rounds to bf16 exactly where the library stores
  bf16 (normed rows, q/k/v, attention out, residual stream, gate/up below 512
  rows, SiLU-gate).
  Logits agree within atol 2e-2 + rtol 2e-2 (accumulation order only).
* `fp32`: no intermediate rounding. Softmax probabilities agree within 2e-2
  absolute, the bf16 tolerance of the attention path.
Plus a cache round trip: prefill a prompt, decode one more token through the
paged cache the prefill wrote, and compare with prefilling the longer prompt.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BS = 16
FUSED_MLP_ROWS = 512  # zl_decoder_step's threshold for the fused gate/up + SiLU-gate kernel


def _cfg(layers=2):
    from zealot_b200.decoder import DecoderConfig
    return DecoderConfig(num_layers=layers, hidden=512, num_heads=4, num_kv_heads=2, head_dim=128,
                         intermediate=1024, vocab=1000)


def _rmsnorm(x, w, eps):
    import torch
    return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps) * w.float()


def _attend(q, k, v, scale, causal):
    """q [L][H][d], k/v [S][Hkv][d] fp32; grouped GQA (kv head = h // (H/Hkv))."""
    import torch
    H, Hkv = q.shape[1], k.shape[1]
    k = k.repeat_interleave(H // Hkv, dim=1)
    v = v.repeat_interleave(H // Hkv, dim=1)
    s = torch.einsum("lhd,shd->hls", q, k) * scale
    if causal:
        L, S = q.shape[0], k.shape[0]
        mask = torch.ones(L, S, dtype=torch.bool, device=q.device).triu(S - L + 1)
        s = s.masked_fill(mask, float("-inf"))
    return torch.einsum("hls,shd->lhd", torch.softmax(s, -1), v)


def reference_step(cfg, w, batch, k_pools, v_pools, round_bf16=True):
    """Returns fp32 logits [num_last][vocab]; k_pools / v_pools are fp32 copies of
    the device pools and are updated with this step's K/V."""
    import torch
    bf = (lambda t: t.to(torch.bfloat16).float()) if round_bf16 else (lambda t: t)
    H, Hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    scale = 1.0 / np.sqrt(d)
    toks = batch.tokens.long()
    slots = batch.slot_mapping.long()
    cu = batch.cu_prefill.cpu().numpy()
    P = batch.prefill_tokens
    tables = batch.block_tables.cpu().numpy()
    lens = batch.seq_lens.cpu().numpy()
    x = w["embed"].float()[toks]
    for l, lw in enumerate(w["layers"]):
        h = bf(_rmsnorm(x, lw["attn_norm"], cfg.rms_eps))
        q = bf(h @ lw["wq"].float().T).view(-1, H, d)
        k = bf(h @ lw["wk"].float().T).view(-1, Hkv, d)
        v = bf(h @ lw["wv"].float().T).view(-1, Hkv, d)
        kp, vp = k_pools[l], v_pools[l]
        blk, off = slots // BS, slots % BS
        kp[blk, :, off] = k
        vp[blk, :, off] = v
        o = torch.zeros_like(q)
        for i in range(batch.num_prefill):
            a, b = int(cu[i]), int(cu[i + 1])
            o[a:b] = _attend(q[a:b], k[a:b], v[a:b], scale, True)
        for i in range(batch.num_decode):
            n = int(lens[i])
            ids = torch.as_tensor(tables[i][: (n + BS - 1) // BS], device=q.device).long()
            kk = kp[ids].permute(0, 2, 1, 3).reshape(-1, Hkv, d)[:n]
            vv = vp[ids].permute(0, 2, 1, 3).reshape(-1, Hkv, d)[:n]
            o[P + i: P + i + 1] = _attend(q[P + i: P + i + 1], kk, vv, scale, False)
        o = bf(o).view(-1, H * d)
        x = bf(x + o @ lw["wo"].float().T)
        h = bf(_rmsnorm(x, lw["mlp_norm"], cfg.rms_eps))
        # steps of FUSED_MLP_ROWS rows or more take silu(g) * u from the fp32
        # accumulators (zl_linear_swiglu): gate/up is not rounded there
        gu = h @ lw["w_gate_up"].float().T
        if x.shape[0] < FUSED_MLP_ROWS:
            gu = bf(gu)
        g, u = gu[:, : cfg.intermediate], gu[:, cfg.intermediate:]
        act = bf(torch.nn.functional.silu(g) * u)
        x = bf(x + act @ lw["w_down"].float().T)
    last = bf(_rmsnorm(x[batch.last_rows.long()], w["final_norm"], cfg.rms_eps))
    return last @ w["lm_head"].float().T


def _mixed_case(cfg, seed, prefill_lens, decode_lens, num_blocks=256):
    """Prefill chunks on fresh blocks plus decode sequences whose earlier positions
    hold random K/V (as if computed by earlier steps)."""
    import torch
    from zealot_b200.decoder import StepBatch
    rng = np.random.default_rng(seed)
    perm = list(rng.permutation(num_blocks))
    pre_tables = []
    for L in prefill_lens:
        n = (L + BS - 1) // BS
        pre_tables.append([int(perm.pop()) for _ in range(n)])
    mb = max([(n + BS - 1) // BS for n in decode_lens] + [1])
    dtab = np.full((len(decode_lens), mb), -1, np.int32)
    for i, n in enumerate(decode_lens):
        for j in range((n + BS - 1) // BS):
            dtab[i, j] = perm.pop()
    chunks = [rng.integers(0, cfg.vocab, L) for L in prefill_lens]
    dtoks = rng.integers(0, cfg.vocab, len(decode_lens))
    batch = StepBatch.build(chunks, dtoks, dtab, decode_lens, pre_tables, BS)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    shape = (num_blocks, cfg.num_kv_heads, BS, cfg.head_dim)
    kps = [torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
           for _ in range(cfg.num_layers)]
    vps = [torch.randn(shape, generator=g, device="cuda").to(torch.bfloat16)
           for _ in range(cfg.num_layers)]
    return batch, kps, vps


@pytest.mark.parametrize("prefill_lens,decode_lens", [
    ([200, 129, 64], [300, 17, 1000, 1, 513]),  # mixed step, ragged chunks and contexts
    ([333], []),                                # prefill only
    ([600, 300], [40, 900]),                    # 902 rows: fused gate/up + SiLU-gate
    ([], [40, 700, 128]),                       # decode only
])
def test_decoder_step_matches_torch(ctx, prefill_lens, decode_lens):
    import torch
    from zealot_b200.decoder import Decoder, random_weights
    cfg = _cfg()
    w = random_weights(cfg, seed=3)
    dec = Decoder(ctx, cfg, w)
    batch, kps, vps = _mixed_case(cfg, 11, prefill_lens, decode_lens)
    k32 = [t.float() for t in kps]
    v32 = [t.float() for t in vps]
    k32b = [t.clone() for t in k32]
    v32b = [t.clone() for t in v32]
    logits = dec.step(batch, kps, vps, BS)
    ctx.check_status()
    ref = reference_step(cfg, w, batch, k32, v32, round_bf16=True)
    torch.testing.assert_close(logits, ref, atol=2e-2, rtol=2e-2)
    # the step wrote this step's K/V into the pools at the slot mapping
    for l in range(cfg.num_layers):
        torch.testing.assert_close(kps[l].float(), k32[l], atol=2e-2, rtol=2e-2)
        torch.testing.assert_close(vps[l].float(), v32[l], atol=2e-2, rtol=2e-2)
    ref32 = reference_step(cfg, w, batch, k32b, v32b, round_bf16=False)
    dp = (torch.softmax(logits, -1) - torch.softmax(ref32, -1)).abs().max().item()
    assert dp <= 2e-2, dp


def test_decoder_prefill_then_decode_round_trip(ctx):
    """Decode of token L through the paged cache written by the prefill of tokens
    0..L-1 equals the last row of a prefill over tokens 0..L (bf16 tolerance)."""
    import torch
    from zealot_b200.decoder import Decoder, StepBatch, random_weights
    cfg = _cfg(layers=3)
    w = random_weights(cfg, seed=5)
    dec = Decoder(ctx, cfg, w)
    rng = np.random.default_rng(2)
    L = 150
    ids = rng.integers(0, cfg.vocab, L + 1)
    nb = (L + 1 + BS - 1) // BS
    table = list(rng.permutation(64)[:nb])
    kps, vps = dec.new_pools(64, BS)
    first = StepBatch.build([ids[:L]], [], np.zeros((0, 1), np.int32), [], [table], BS)
    dec.step(first, kps, vps, BS)
    dtab = np.asarray([table], np.int32)
    second = StepBatch.build([], [ids[L]], dtab, [L + 1], [], BS)
    got = dec.step(second, kps, vps, BS)
    k2, v2 = dec.new_pools(64, BS)
    whole = StepBatch.build([ids], [], np.zeros((0, 1), np.int32), [], [table], BS)
    want = dec.step(whole, k2, v2, BS)
    ctx.check_status()
    torch.testing.assert_close(got, want, atol=3e-2, rtol=3e-2)
    assert int(got.argmax()) == int(want.argmax())


def test_decoder_rejects_bad_arguments(ctx):
    import zealot_b200 as zb
    from zealot_b200.decoder import Decoder, random_weights
    cfg = _cfg(layers=1)
    w = random_weights(cfg, seed=1)
    dec = Decoder(ctx, cfg, w)
    batch, kps, vps = _mixed_case(cfg, 1, [16], [20])
    with pytest.raises(zb.InvalidArgument):
        dec.step(batch, kps[:0], vps[:0], BS)
    bad = dict(w)
    bad["layers"] = [dict(w["layers"][0], wq=w["layers"][0]["wq"][:, :256].contiguous())]
    with pytest.raises(zb.InvalidArgument):
        Decoder(ctx, cfg, bad)
