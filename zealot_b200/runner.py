"""CudaModelRunner behind the engine's ModelRunner boundary (src/engine.rs:15-47).

`Sequence` carries exactly what the reference runner reads from
src/scheduler.rs:11-113 (request_id, step_input(), is_prefill(), prefill_pos);
`StepOut` is src/engine.rs:39-47. The runner returns logits and leaves
sampling to the engine, as the CPU runner does (model_runner_cpu.rs:267-272).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _capi
from .context import GpuContext, GQA_MODULO
from .errors import check


@dataclass
class Sequence:
    """The runner-visible part of scheduler.rs:11-113."""
    request_id: str
    prompt_tokens: list
    output_tokens: list = field(default_factory=list)
    prefill_pending: bool = True
    prefill_pos: int = 0
    chunk_size: int = 0

    def step_input(self) -> list:
        """scheduler.rs:88-101."""
        if self.prefill_pending:
            end = min(self.prefill_pos + self.chunk_size, len(self.prompt_tokens))
            return list(self.prompt_tokens[self.prefill_pos:end]) + list(self.output_tokens)
        return [self.output_tokens[-1]]

    def is_prefill(self) -> bool:
        return self.prefill_pending


@dataclass
class StepOut:
    request_id: str
    token: int | None
    logits: np.ndarray | None
    text: str | None = None


class CudaModelRunner:
    """zl_runner: layer-0 attention model of the CPU runner, on the GPU with a paged KV cache."""

    def __init__(self, ctx: GpuContext, weights: dict, num_gpu_blocks: int = 1024,
                 block_size: int = 16, max_blocks_per_seq: int | None = None,
                 gqa_map: int = GQA_MODULO):
        self.ctx = ctx
        self.lib = ctx.lib
        w = {k: np.ascontiguousarray(weights[k], dtype=np.float32)
             for k in ("embedding", "q_proj", "k_proj", "v_proj", "attn_proj", "lm_head")}
        self._w = w  # host copies stay alive for the duration of create
        self.vocab_size = int(weights["vocab_size"])
        cfg = _capi.zl_runner_cfg(
            int(weights["hidden_dim"]), int(weights["num_heads"]), int(weights["num_kv_heads"]),
            int(weights["head_dim"]), int(weights.get("num_layers", 1)), self.vocab_size,
            num_gpu_blocks, block_size, max_blocks_per_seq or num_gpu_blocks, gqa_map)
        fp = ctypes.POINTER(ctypes.c_float)
        cw = _capi.zl_runner_weights(*(w[k].ctypes.data_as(fp) for k in
                                       ("embedding", "q_proj", "k_proj", "v_proj", "attn_proj", "lm_head")))
        h = ctypes.c_void_p()
        check(self.lib.zl_runner_create(ctx.handle, ctypes.byref(cfg), ctypes.byref(cw), ctypes.byref(h)))
        self.handle = h

    def step(self, batch: list) -> list:
        """ModelRunner::step: one forward step for every sequence of the batch."""
        n = len(batch)
        if n == 0:
            return []
        arr = (_capi.zl_seq_input * n)()
        keep = []
        for i, s in enumerate(batch):
            toks = np.ascontiguousarray(s.step_input(), dtype=np.int64)
            rid = s.request_id.encode()
            keep.append((toks, rid))
            arr[i] = _capi.zl_seq_input(rid, toks.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                        toks.size, int(s.is_prefill()), int(s.prefill_pos))
        logits = np.empty((n, self.vocab_size), np.float32)
        check(self.lib.zl_runner_step(self.handle, arr, n,
                                      logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        return [StepOut(s.request_id, None, logits[i].copy()) for i, s in enumerate(batch)]

    def drop_state(self, request_id: str) -> None:
        check(self.lib.zl_runner_drop_state(self.handle, request_id.encode()))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.zl_runner_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
