"""Writes the golden fixtures under tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

gqa_step.npz  -- logits of the reference's own runner fixture
                 (src/model_runner_cpu.rs:366-400: weights (i % 7) / 7, prompt [1, 2, 3]).
c1_greedy.npz -- config C1 (random-init GPT-2-style, d_model 32, 4 heads x 8, vocab 1000,
                 N(0, 0.02) weights, seed 1234): 4 prompts of 32 ids, 32 greedy tokens from
                 the CPU runner in recompute form (src/scheduler.rs:129-133), final-step logits.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle  # noqa: E402


def gqa_weights():
    rand = lambda n: (np.arange(n) % 7).astype(np.float32) / np.float32(7.0)
    return dict(hidden_dim=8, num_heads=4, num_kv_heads=2, head_dim=2, vocab_size=4,
                embedding=rand(4 * 8), q_proj=rand(8 * 8), k_proj=rand(8 * 4), v_proj=rand(8 * 4),
                attn_proj=rand(8 * 8), lm_head=rand(8 * 4))


def c1_weights(seed=1234):
    rng = np.random.default_rng(seed)
    hid, H, d, V = 32, 4, 8, 1000
    n = lambda *s: rng.normal(0.0, 0.02, size=s).astype(np.float32)
    return dict(hidden_dim=hid, num_heads=H, num_kv_heads=H, head_dim=d, vocab_size=V, num_layers=5,
                embedding=n(V, hid), q_proj=n(hid, H * d), k_proj=n(hid, H * d), v_proj=n(hid, H * d),
                attn_proj=n(hid, hid), lm_head=n(hid, V))


def c1_prompts(seed=1234, n=4, L=32, vocab=1000):
    rng = np.random.default_rng(seed + 1)
    return rng.integers(0, vocab, size=(n, L)).astype(np.int64)


def c1_greedy(w, prompts, steps=32):
    toks = np.zeros((len(prompts), steps), np.int64)
    last = np.zeros((len(prompts), w["vocab_size"]), np.float32)
    for i, p in enumerate(prompts):
        hist = list(p)
        for t in range(steps):
            logits = oracle.runner_step(w, hist)
            tok = oracle.argmax(logits)
            toks[i, t] = tok
            hist.append(tok)
            last[i] = logits
    return toks, last


def main():
    np.savez(os.path.join(HERE, "gqa_step.npz"), logits=oracle.runner_step(gqa_weights(), [1, 2, 3]))
    w = c1_weights()
    prompts = c1_prompts()
    toks, last = c1_greedy(w, prompts)
    np.savez(os.path.join(HERE, "c1_greedy.npz"), prompts=prompts, tokens=toks, last_logits=last)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
