"""Full-decoder engine step: the layer loop of CudaModelRunner::step
(src/cuda_runner.rs:303-607) batched over all sequences of a step.

`Decoder` holds the bf16 weights (torch tensors as device buffers) and calls
`zl_decoder_step`, which runs RMSNorm, the q/k/v, o, gate/up and down GEMMs
(cuBLAS, fp32 accumulate, residual add folded into the GEMM), SiLU-gate,
`reshape_and_cache`, varlen causal prefill and paged decode for every layer,
then the final RMSNorm and lm_head on the requested rows.

`StepBatch.build` lays out one step the way the engine schedules it
(src/scheduler.rs:88-113): prefill chunks first, packed back to back, then one
row per decode sequence.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _capi
from .context import GpuContext, ptr
from .errors import check, InvalidArgument


@dataclass(frozen=True)
class DecoderConfig:
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float = 1e-6  # the reference runner's launch_rms_norm_raw eps (cuda_runner.rs:323)

    @staticmethod
    def mistral_7b() -> "DecoderConfig":
        return DecoderConfig(32, 4096, 32, 8, 128, 14336, 32000)

    def layer_shapes(self) -> dict[str, tuple[int, ...]]:
        H, Hkv, d, hid, inter = (self.num_heads, self.num_kv_heads, self.head_dim, self.hidden,
                                 self.intermediate)
        return {"attn_norm": (hid,), "wq": (H * d, hid), "wk": (Hkv * d, hid),
                "wv": (Hkv * d, hid), "wo": (hid, H * d), "mlp_norm": (hid,),
                "w_gate_up": (2 * inter, hid), "w_down": (hid, inter)}


def random_weights(cfg: DecoderConfig, seed: int = 0, device: str = "cuda", std: float = 0.02):
    """Seeded random bf16 weights of the architecture (no checkpoint): N(0, std)
    matrices and norm weights around 1."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def mat(*shape):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std).to(
            torch.bfloat16)

    def norm(n):
        return (1.0 + 0.1 * torch.randn((n,), generator=g, device=device)).to(torch.bfloat16)

    layers = []
    for _ in range(cfg.num_layers):
        lw = {k: (norm(s[0]) if len(s) == 1 else mat(*s)) for k, s in cfg.layer_shapes().items()}
        # q, k and v projections back to back in one buffer (row slices of it): a step
        # with few rows then reads the three with one GEMM (zl_decoder_step)
        qkv = torch.cat([lw["wq"], lw["wk"], lw["wv"]])
        nq, nk = lw["wq"].shape[0], lw["wk"].shape[0]
        lw["wq"], lw["wk"], lw["wv"] = qkv[:nq], qkv[nq:nq + nk], qkv[nq + nk:]
        layers.append(lw)
    return {"embed": mat(cfg.vocab, cfg.hidden) * 50, "layers": layers,
            "final_norm": norm(cfg.hidden), "lm_head": mat(cfg.vocab, cfg.hidden)}


@dataclass
class StepBatch:
    """Device tensors of one step; see zl_step_batch in include/zealot_attn.h."""
    tokens: object
    slot_mapping: object
    cu_prefill: object
    num_prefill: int
    max_prefill_len: int
    prefill_tokens: int
    block_tables: object
    seq_lens: object
    num_decode: int
    max_blocks_per_seq: int
    last_rows: object

    @staticmethod
    def build(prefill_chunks, decode_tokens, decode_tables, decode_lens, prefill_tables,
              block_size: int, device="cuda") -> "StepBatch":
        """prefill_chunks: list of int token arrays (whole prompts, position 0..L-1),
        prefill_tables: their block-id lists; decode_tokens: one id per decode
        sequence whose K/V goes to position decode_lens[i]-1; decode_tables: [B][max]
        int32, -1 padded. Returns the batch with last_rows = the last row of every
        prefill chunk, then every decode row."""
        import torch
        toks, slots, cu = [], [], [0]
        for ids, table in zip(prefill_chunks, prefill_tables):
            L = len(ids)
            pos = np.arange(L)
            slots.append(np.asarray(table, np.int64)[pos // block_size] * block_size
                         + pos % block_size)
            toks.append(np.asarray(ids, np.int64))
            cu.append(cu[-1] + L)
        P = cu[-1]
        dt = (np.asarray(decode_tables, np.int32).reshape(len(decode_tokens), -1)
              if len(decode_tokens) else np.zeros((0, 1), np.int32))
        dl = np.asarray(decode_lens, np.int32)
        if len(decode_tokens):
            pos = dl.astype(np.int64) - 1
            slots.append(dt[np.arange(len(dl)), pos // block_size].astype(np.int64) * block_size
                         + pos % block_size)
            toks.append(np.asarray(decode_tokens, np.int64))
        last = np.concatenate([np.asarray(cu[1:], np.int32) - 1,
                               P + np.arange(len(decode_tokens), dtype=np.int32)])

        def dev(a, dtype):
            return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)

        return StepBatch(
            tokens=dev(np.concatenate(toks) if toks else np.zeros(0, np.int64), torch.int64),
            slot_mapping=dev(np.concatenate(slots) if slots else np.zeros(0, np.int64),
                             torch.int64),
            cu_prefill=dev(np.asarray(cu, np.int32), torch.int32),
            num_prefill=len(prefill_chunks),
            max_prefill_len=max((len(c) for c in prefill_chunks), default=0),
            prefill_tokens=P,
            block_tables=dev(dt if dt.size else np.zeros((0, 1), np.int32), torch.int32),
            seq_lens=dev(dl, torch.int32), num_decode=len(decode_tokens),
            max_blocks_per_seq=int(dt.shape[1]) if dt.ndim == 2 and dt.size else 1,
            last_rows=dev(last, torch.int32))

    @property
    def num_last(self) -> int:
        return int(self.last_rows.numel())

    def as_c(self) -> _capi.zl_step_batch:
        return _capi.zl_step_batch(
            ptr(self.tokens), ptr(self.slot_mapping), ptr(self.cu_prefill), self.num_prefill,
            self.max_prefill_len, self.prefill_tokens, ptr(self.block_tables), ptr(self.seq_lens),
            self.num_decode, self.max_blocks_per_seq, ptr(self.last_rows), self.num_last)


class Decoder:
    """A decoder model resident on one GPU; `step` runs one engine step."""

    def __init__(self, ctx: GpuContext, cfg: DecoderConfig, weights: dict):
        import torch
        self.ctx, self.cfg, self.w = ctx, cfg, weights
        for name, t in [("embed", weights["embed"]), ("final_norm", weights["final_norm"]),
                        ("lm_head", weights["lm_head"])]:
            if t.dtype != torch.bfloat16 or not t.is_contiguous() or not t.is_cuda:
                raise InvalidArgument(f"{name} must be a contiguous bf16 cuda tensor")
        shapes = cfg.layer_shapes()
        self._layers = (_capi.zl_layer_weights * cfg.num_layers)()
        for i, lw in enumerate(weights["layers"]):
            for k, s in shapes.items():
                t = lw[k]
                if tuple(t.shape) != s or t.dtype != torch.bfloat16 or not t.is_contiguous():
                    raise InvalidArgument(f"layer {i} {k}: want contiguous bf16 {s}")
                setattr(self._layers[i], k, ptr(t))
        self._model = _capi.zl_decoder(
            cfg.num_layers, cfg.hidden, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
            cfg.intermediate, cfg.vocab, cfg.rms_eps, ptr(weights["embed"]),
            self._layers, ptr(weights["final_norm"]), ptr(weights["lm_head"]))

    def new_pools(self, num_blocks: int, block_size: int, device="cuda"):
        """Per-layer K and V pools [num_blocks][Hkv][block_size][d] bf16 (zeroed)."""
        import torch
        shape = (num_blocks, self.cfg.num_kv_heads, block_size, self.cfg.head_dim)
        k = [torch.zeros(shape, dtype=torch.bfloat16, device=device)
             for _ in range(self.cfg.num_layers)]
        v = [torch.zeros(shape, dtype=torch.bfloat16, device=device)
             for _ in range(self.cfg.num_layers)]
        return k, v

    def step(self, batch: StepBatch, k_pools, v_pools, block_size: int, logits=None,
             stream=None):
        """Runs one step; returns fp32 logits [num_last][vocab] on the device."""
        import torch
        L = self.cfg.num_layers
        if len(k_pools) != L or len(v_pools) != L:
            raise InvalidArgument(f"need {L} K and V pools")
        num_blocks = k_pools[0].shape[0]
        if logits is None:
            logits = torch.empty((batch.num_last, self.cfg.vocab), dtype=torch.float32,
                                 device=batch.tokens.device)
        kp = (ctypes.c_void_p * L)(*[ptr(t) for t in k_pools])
        vp = (ctypes.c_void_p * L)(*[ptr(t) for t in v_pools])
        cb = batch.as_c()
        check(self.ctx.lib.zl_decoder_step(self.ctx.handle, ctypes.byref(self._model), kp, vp,
                                           num_blocks, block_size, ctypes.byref(cb), ptr(logits),
                                           self.ctx.stream(stream)))
        return logits


class DecodeGraph:
    """Device-resident decode loop (zl_decode_graph_*): `rows` decode slots whose
    tokens, lengths, block tables, sampling parameters and output-token counts
    stay on the device; one step is one CUDA-graph launch (use_graph=False issues
    the same launches eagerly). Block ids come from the caller's BlockManager."""

    def __init__(self, dec: Decoder, k_pools, v_pools, block_size: int, rows: int,
                 max_blocks_per_seq: int, use_graph: bool = True):
        self.dec, self.ctx, self.rows = dec, dec.ctx, rows
        self._pools = (list(k_pools), list(v_pools))  # kept alive with the graph
        L = dec.cfg.num_layers
        kp = (ctypes.c_void_p * L)(*[ptr(t) for t in k_pools])
        vp = (ctypes.c_void_p * L)(*[ptr(t) for t in v_pools])
        h = ctypes.c_void_p()
        check(self.ctx.lib.zl_decode_graph_create(
            self.ctx.handle, ctypes.byref(dec._model), kp, vp, k_pools[0].shape[0], block_size, rows,
            max_blocks_per_seq, int(use_graph), ctypes.byref(h)))
        self.handle = h
        self._tok = np.zeros(rows, np.int64)
        self._lp = np.zeros(rows, np.float32)

    def set_row(self, row: int, block_ids, seq_len: int, next_token: int, params=None, history=()):
        from .sampling import SamplingParams
        p = params or SamplingParams()
        cp = _capi.zl_sampling_params(p.temperature, p.top_k, p.top_p, p.repetition_penalty,
                                      p.frequency_penalty, p.presence_penalty)
        b = np.ascontiguousarray(block_ids, np.int32)
        hist = np.ascontiguousarray(history, np.int64)
        check(self.ctx.lib.zl_decode_graph_set_row(
            self.handle, row, b.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), b.size, seq_len,
            int(next_token), ctypes.byref(cp), hist.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
            hist.size))

    def clear_row(self, row: int):
        check(self.ctx.lib.zl_decode_graph_clear_row(self.handle, row))

    def rows_needing_block(self) -> list:
        out = np.zeros(self.rows, np.int32)
        n = ctypes.c_int()
        check(self.ctx.lib.zl_decode_graph_rows_needing_block(
            self.handle, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.byref(n)))
        return out[: n.value].tolist()

    def step(self, new_blocks: dict, uniforms, stream=None):
        """new_blocks: {row: block id} for every row in rows_needing_block()."""
        nb = np.asarray(sorted(new_blocks.items()), np.int32).reshape(-1, 2)
        u = np.ascontiguousarray(uniforms, np.float32)
        if u.size != self.rows:
            raise InvalidArgument(f"need {self.rows} uniforms")
        check(self.ctx.lib.zl_decode_graph_step(
            self.handle, nb.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), nb.shape[0],
            u.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
            0 if stream is None else self.ctx.stream(stream)))

    def tokens(self):
        """Waits for the last step; (token ids int64 [rows], logprobs float32 [rows])."""
        check(self.ctx.lib.zl_decode_graph_tokens(
            self.handle, self._tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
            self._lp.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        return self._tok.copy(), self._lp.copy()

    def logits(self):
        """Waits for the last step; the logits it sampled from, float32 [rows][vocab]."""
        out = np.empty((self.rows, self.dec.cfg.vocab), np.float32)
        check(self.ctx.lib.zl_decode_graph_logits(self.handle,
                                                  out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        return out

    @property
    def num_kernels(self) -> int:
        return int(self.ctx.lib.zl_decode_graph_num_kernels(self.handle))

    def close(self):
        if self.handle:
            check(self.ctx.lib.zl_decode_graph_destroy(self.handle))
            self.handle = None
