"""CudaAttention: the attention operators of the hot path.

Mirrors src/attention/cuda.rs:20-210 of the reference (paged_forward,
forward_gpu) plus the KV scatter that replaced KVCache::store_kv's copies.
Arguments keep the reference's names and meaning; tensors are torch device
tensors, checked here and handed to the C ABI by address.
"""
from __future__ import annotations

from .context import GpuContext, GQA_GROUPED, dtype_code, ptr
from .errors import check, InvalidArgument


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise InvalidArgument(msg)


class CudaAttention:
    def __init__(self, ctx: GpuContext):
        self.ctx = ctx
        self.lib = ctx.lib

    # ------------------------------------------------------------ KV scatter
    def reshape_and_cache(self, k, v, k_pool, v_pool, slot_mapping, num_kv_heads: int,
                          head_dim: int, block_size: int, num_blocks: int, stream=None) -> None:
        """k, v [T][Hkv][d] -> pools [num_blocks][Hkv][bs][d] at slot_mapping[T] (int64)."""
        import torch
        _need(k.dtype == v.dtype == k_pool.dtype == v_pool.dtype, "dtype mismatch")
        _need(slot_mapping.dtype == torch.int64, "slot_mapping must be int64")
        for t in (k, v, k_pool, v_pool, slot_mapping):
            _need(t.is_contiguous() and t.is_cuda, "tensors must be contiguous CUDA tensors")
        T = slot_mapping.numel()
        _need(k.numel() == T * num_kv_heads * head_dim and v.numel() == k.numel(), "k/v shape")
        _need(k_pool.numel() >= num_blocks * block_size * num_kv_heads * head_dim, "pool too small")
        check(self.lib.zl_reshape_and_cache(self.ctx.handle, ptr(k), ptr(v), ptr(k_pool), ptr(v_pool),
                                            ptr(slot_mapping), T, num_kv_heads, head_dim, block_size,
                                            num_blocks, dtype_code(k.dtype), self.ctx.stream(stream)))

    # ----------------------------------------------------------- paged decode
    def paged_forward(self, q, k_pool, v_pool, block_tables, seq_lens, o, num_seqs: int,
                      num_heads: int, num_kv_heads: int, head_dim: int, block_size: int,
                      max_blocks_per_seq: int, num_blocks: int | None = None, scale: float = 0.0,
                      gqa_map: int = GQA_GROUPED, num_splits: int = 0, stream=None) -> None:
        """CudaAttention::paged_forward (cuda.rs:126-210): q/o [B][H][d], block_tables
        [B][max_blocks] int32 (negative = end), seq_lens [B] int32."""
        import torch
        _need(q.dtype == k_pool.dtype == v_pool.dtype == o.dtype, "dtype mismatch")
        _need(block_tables.dtype == torch.int32 and seq_lens.dtype == torch.int32, "int32 tables")
        for t in (q, k_pool, v_pool, block_tables, seq_lens, o):
            _need(t.is_contiguous() and t.is_cuda, "tensors must be contiguous CUDA tensors")
        _need(q.numel() == num_seqs * num_heads * head_dim and o.numel() == q.numel(), "q/o shape")
        _need(block_tables.numel() >= num_seqs * max_blocks_per_seq, "block_tables shape")
        per_block = block_size * num_kv_heads * head_dim
        if num_blocks is None:
            num_blocks = k_pool.numel() // per_block
        _need(k_pool.numel() >= num_blocks * per_block, "pool smaller than num_blocks")
        check(self.lib.zl_paged_decode(self.ctx.handle, ptr(q), ptr(k_pool), ptr(v_pool),
                                       ptr(block_tables), ptr(seq_lens), ptr(o), num_seqs, num_heads,
                                       num_kv_heads, head_dim, block_size, max_blocks_per_seq,
                                       num_blocks, scale, gqa_map, num_splits, dtype_code(q.dtype),
                                       self.ctx.stream(stream)))

    def paged_forward_partial(self, q, k_pool, v_pool, block_tables, tok_begin, tok_end, m, l, o,
                              num_seqs: int, num_heads: int, num_kv_heads: int, head_dim: int,
                              block_size: int, max_blocks_per_seq: int, num_blocks: int | None = None,
                              scale: float = 0.0, gqa_map: int = GQA_GROUPED, stream=None) -> None:
        """Unnormalised (m, l, o) over tokens [tok_begin, tok_end) of each sequence."""
        import torch
        _need(m.dtype == l.dtype == o.dtype == torch.float32, "partials are float32")
        per_block = block_size * num_kv_heads * head_dim
        if num_blocks is None:
            num_blocks = k_pool.numel() // per_block
        check(self.lib.zl_paged_decode_partial(
            self.ctx.handle, ptr(q), ptr(k_pool), ptr(v_pool), ptr(block_tables), ptr(tok_begin),
            ptr(tok_end), ptr(m), ptr(l), ptr(o), num_seqs, num_heads, num_kv_heads, head_dim,
            block_size, max_blocks_per_seq, num_blocks, scale, gqa_map, dtype_code(q.dtype),
            self.ctx.stream(stream)))

    def merge_partials(self, m, l, o, out, stream=None) -> None:
        """m, l [P][rows], o [P][rows][d] float32 -> out [rows][d]."""
        P = m.shape[0]
        rows = m[0].numel()
        d = o.shape[-1]
        check(self.lib.zl_merge_partials(self.ctx.handle, ptr(m), ptr(l), ptr(o), P, rows, d,
                                         ptr(out), dtype_code(out.dtype), self.ctx.stream(stream)))

    # ---------------------------------------------------------------- prefill
    def forward_gpu(self, q, k, v, cu_seqlens, o, num_heads: int, num_kv_heads: int,
                    head_dim: int, max_seq_len: int, causal: bool = True, scale: float = 0.0,
                    gqa_map: int = GQA_GROUPED, stream=None) -> None:
        """Varlen form of CudaAttention::forward_gpu (cuda.rs:56-110): q/o [T][H][d],
        k/v [T][Hkv][d], cu_seqlens [n+1] int32."""
        import torch
        _need(q.dtype == k.dtype == v.dtype == o.dtype, "dtype mismatch")
        _need(cu_seqlens.dtype == torch.int32, "cu_seqlens must be int32")
        for t in (q, k, v, cu_seqlens, o):
            _need(t.is_contiguous() and t.is_cuda, "tensors must be contiguous CUDA tensors")
        n = cu_seqlens.numel() - 1
        T = q.shape[0]
        _need(q.numel() == T * num_heads * head_dim and k.numel() == T * num_kv_heads * head_dim
              and v.numel() == k.numel() and o.numel() == q.numel(), "q/k/v/o shapes")
        check(self.lib.zl_prefill_varlen(self.ctx.handle, ptr(q), ptr(k), ptr(v), ptr(cu_seqlens), n,
                                         max_seq_len, T, ptr(o), num_heads, num_kv_heads, head_dim, scale,
                                         int(causal), gqa_map, dtype_code(q.dtype),
                                         self.ctx.stream(stream)))
