"""GPU sampling for a whole step: the Python mirror of Sampler / SamplingParams
(src/sampling.rs:22-230) over `zl_sample`.

One call samples every row of a [rows][vocab] fp32 logits tensor on the device:
the allowed-token mask, greedy fast path, temperature, presence / frequency /
repetition penalties, top-k, top-p and the multinomial draw run in one kernel
launch, and only the token ids (8 bytes per row) need to come back to the host,
instead of the vocab-sized logits row per sequence the engine copies today
(src/cuda_runner.rs:645). The engine keeps its RNG (per-request StdRng,
src/engine.rs:157-164): it passes each row's draw r in [0, 1).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _capi
from .context import GpuContext, ptr
from .errors import check, InvalidArgument

SAMPLE_ALL_MASKED = 1  # SamplingError::AllTokensMasked (token 0, logprob -inf)
SAMPLE_FELL_BACK = 2   # the mask left nothing; sampled unconstrained (engine.rs:190-206)


@dataclass
class SamplingParams:
    """src/sampling.rs:22-45 (defaults mean no-op). The seed stays with the caller's RNG."""
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 0.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0


@dataclass
class SampledTokens:
    token_ids: object   # int64 [rows] (device)
    logprobs: object    # float32 [rows] (device)
    status: object      # int32 [rows] (device), SAMPLE_* bits


@dataclass
class SamplerBatch:
    """Device-side inputs of one zl_sample call, built once by GpuSampler.prepare."""
    rows: int
    vocab: int
    params: object
    allowed_bits: object
    mask_rows: object
    mask_len: int
    pen_off: object
    pen_ids: object
    pen_cnt: object


class GpuSampler:
    def __init__(self, ctx: GpuContext):
        self.ctx = ctx

    def prepare(self, rows: int, vocab: int, params, prev_outputs=None, masks=None,
                device="cuda") -> SamplerBatch:
        """Packs per-row params, penalty lists (distinct in-range previous ids with
        their counts: the frequency map of sampling.rs:130-134) and allowed-token
        bitmasks, and copies them to the device."""
        import torch
        if isinstance(params, SamplingParams):
            params = [params] * rows
        if len(params) != rows:
            raise InvalidArgument(f"{len(params)} sampling params for {rows} rows")
        arr = (_capi.zl_sampling_params * max(rows, 1))()
        for i, p in enumerate(params):
            arr[i] = _capi.zl_sampling_params(p.temperature, p.top_k, p.top_p, p.repetition_penalty,
                                              p.frequency_penalty, p.presence_penalty)
        raw = np.frombuffer(bytes(arr), dtype=np.uint8)
        d_params = torch.from_numpy(raw.copy()).to(device)
        d_off = d_ids = d_cnt = None
        if prev_outputs is not None and any(len(p if p is not None else ()) for p in prev_outputs):
            off, ids, cnt = [0], [], []
            for p in prev_outputs:
                a = np.asarray(p if p is not None else [], dtype=np.int64)
                a = a[(a >= 0) & (a < vocab)]
                u, c = np.unique(a, return_counts=True)
                ids.append(u)
                cnt.append(c.astype(np.int32))
                off.append(off[-1] + u.size)
            d_off = torch.from_numpy(np.asarray(off, np.int32)).to(device)
            d_ids = torch.from_numpy(np.concatenate(ids + [np.zeros(1, np.int64)])).to(device)
            d_cnt = torch.from_numpy(np.concatenate(cnt + [np.zeros(1, np.int32)])).to(device)
        d_bits = d_rows = None
        mask_len = 0
        if masks is not None and any(m is not None for m in masks):
            mask_len = max(len(m) for m in masks if m is not None)
            words = (mask_len + 31) // 32
            bits = np.full((rows, words * 32), True)
            use = np.zeros(rows, np.uint8)
            for i, m in enumerate(masks):
                if m is not None:
                    bits[i, : len(m)] = np.asarray(m, dtype=bool)
                    use[i] = 1
            packed = np.packbits(bits, axis=1, bitorder="little").view(np.uint32)
            d_bits = torch.from_numpy(np.ascontiguousarray(packed)).to(device)
            d_rows = torch.from_numpy(use).to(device)
        self._greedy_only = all(p.temperature < 1e-7 for p in params)
        return SamplerBatch(rows, vocab, d_params, d_bits, d_rows, mask_len, d_off, d_ids, d_cnt)

    def launch(self, batch: SamplerBatch, logits, uniforms, out: SampledTokens = None,
               fallback_unmasked: bool = True, dense_counts=None, update_counts: bool = False,
               stream=None) -> SampledTokens:
        """One zl_sample launch over prepared inputs; uniforms: float32 device [rows].
        dense_counts: int32 device [rows][vocab] output-token counts used for the
        penalties instead of the prepared lists; update_counts adds each sampled token."""
        import torch
        if (logits.dtype != torch.float32 or logits.dim() != 2 or not logits.is_contiguous()
                or tuple(logits.shape) != (batch.rows, batch.vocab)):
            raise InvalidArgument("logits must be a contiguous float32 [rows][vocab] tensor")
        dev = logits.device
        if out is None:
            out = SampledTokens(torch.empty(batch.rows, dtype=torch.int64, device=dev),
                                torch.empty(batch.rows, dtype=torch.float32, device=dev),
                                torch.empty(batch.rows, dtype=torch.int32, device=dev))
        check(self.ctx.lib.zl_sample(
            self.ctx.handle, ptr(logits), batch.rows, batch.vocab, ptr(batch.params),
            ptr(batch.allowed_bits), ptr(batch.mask_rows), batch.mask_len, ptr(batch.pen_off),
            ptr(batch.pen_ids), ptr(batch.pen_cnt), ptr(dense_counts), int(update_counts),
            ptr(uniforms), int(fallback_unmasked),
            ptr(out.token_ids), ptr(out.logprobs), ptr(out.status), self.ctx.stream(stream)))
        return out

    def sample(self, logits, params, prev_outputs=None, masks=None, uniforms=None,
               fallback_unmasked: bool = True, stream=None) -> SampledTokens:
        """logits: float32 cuda tensor [rows][vocab]. params: one SamplingParams per row
        (or one for all). prev_outputs: per row the previous output ids (or None).
        masks: per row a bool array of allowed tokens or None (unmasked); a mask
        shorter than the vocab allows the rest (sampling.rs:91-93). uniforms: per
        row the draw r in [0, 1) (required unless every row is greedy)."""
        import torch
        if logits.dtype != torch.float32 or logits.dim() != 2 or not logits.is_contiguous():
            raise InvalidArgument("logits must be a contiguous float32 [rows][vocab] tensor")
        rows, vocab = logits.shape
        batch = self.prepare(rows, vocab, params, prev_outputs, masks, logits.device)
        if uniforms is None:
            if not self._greedy_only:
                raise InvalidArgument("uniforms are required for non-greedy rows")
            uniforms = np.zeros(rows, np.float32)
        d_u = uniforms if hasattr(uniforms, "data_ptr") else torch.from_numpy(
            np.asarray(uniforms, np.float32)).to(logits.device)
        return self.launch(batch, logits, d_u, fallback_unmasked=fallback_unmasked, stream=stream)
