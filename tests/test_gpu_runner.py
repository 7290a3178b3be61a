"""Config C1 end to end: the CUDA runner (paged KV cache) against the CPU runner in
recompute form (src/model_runner_cpu.rs:172-276 on prompt + outputs,
src/scheduler.rs:129-133). Logits within 1e-4 relative at every step; identical
greedy streams (src/sampling.rs:233-243)."""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden import c1_prompts, c1_weights  # noqa: E402


def _engine_loop(runner, prompts, steps, on_logits):
    import zealot_b200 as zb
    seqs = [zb.Sequence(f"req-{i}", list(p), chunk_size=512) for i, p in enumerate(prompts)]
    for t in range(steps):
        outs = runner.step(seqs)
        for s, o in zip(seqs, outs):
            on_logits(t, s, o.logits)
            tok = int(np.argmax(o.logits))  # numpy argmax: first maximum, as sampling.rs
            s.output_tokens.append(tok)
            s.prefill_pending = False
    return seqs


def test_c1_greedy_matches_cpu_runner(ctx, oracle):
    import zealot_b200 as zb
    w = c1_weights()
    prompts = c1_prompts()
    golden = np.load(os.path.join(HERE, "golden", "c1_greedy.npz"))
    runner = zb.CudaModelRunner(ctx, w, num_gpu_blocks=1024, block_size=16)
    worst = [0.0]

    def check(t, s, logits):
        hist = list(s.prompt_tokens) + list(s.output_tokens)
        ref = oracle.runner_step(w, hist)
        err = float(np.max(np.abs(logits - ref)) / np.max(np.abs(ref)))
        worst[0] = max(worst[0], err)
        assert err <= 1e-4, (t, s.request_id, err)

    seqs = _engine_loop(runner, prompts, 32, check)
    toks = np.array([s.output_tokens for s in seqs])
    assert np.array_equal(toks, golden["tokens"])
    for s in seqs:
        runner.drop_state(s.request_id)
    runner.close()


def test_runner_drop_state_and_recompute(ctx, oracle):
    """Preemption (drop_state) then a prefill from position 0 recomputes the same logits."""
    import zealot_b200 as zb
    w = c1_weights()
    p = list(c1_prompts()[0][:20])
    runner = zb.CudaModelRunner(ctx, w, num_gpu_blocks=8, block_size=16)
    s = zb.Sequence("a", p, chunk_size=512)
    first = runner.step([s])[0].logits
    s.output_tokens.append(int(np.argmax(first)))
    s.prefill_pending = False
    second = runner.step([s])[0].logits
    runner.drop_state("a")
    s.prefill_pending = True  # recompute: prompt + outputs (scheduler.rs:374-376)
    again = runner.step([s])[0].logits
    np.testing.assert_allclose(again, second, rtol=1e-5, atol=1e-9)
    # a pool of 8 blocks holds 128 tokens: a 200-token sequence is too long
    big = zb.Sequence("b", list(range(200)), chunk_size=512)
    with pytest.raises(zb.ZealotError):
        runner.step([big])
    runner.close()
