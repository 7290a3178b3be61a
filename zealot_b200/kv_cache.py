"""BlockManager (src/block_manager.rs:41-165) and KVCache (src/kv_cache.rs:51-357)."""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import _capi
from .context import GpuContext, device_view, dtype_code, ptr
from .errors import check


@dataclass(frozen=True)
class BlockHandle:
    """BlockHandle (block_manager.rs:18-24)."""
    block_id: int
    generation: int

    def _c(self):
        return _capi.zl_block_handle(self.block_id, self.generation)


class BlockManager:
    """LIFO block pool with refcounts and generations (block_manager.rs:88-165)."""

    def __init__(self, num_gpu_blocks: int, block_size: int):
        self.lib = _capi.load()
        h = ctypes.c_void_p()
        check(self.lib.zl_block_manager_create(num_gpu_blocks, block_size, ctypes.byref(h)))
        self.handle = h
        self.num_gpu_blocks = num_gpu_blocks
        self.block_size = block_size

    def try_allocate(self) -> BlockHandle:
        out = _capi.zl_block_handle()
        check(self.lib.zl_block_manager_try_allocate(self.handle, ctypes.byref(out)))
        return BlockHandle(int(out.block_id), int(out.generation))

    allocate = try_allocate

    def try_free(self, h: BlockHandle) -> None:
        c = h._c()
        check(self.lib.zl_block_manager_try_free(self.handle, ctypes.byref(c)))

    free = try_free

    def try_reference(self, h: BlockHandle) -> None:
        c = h._c()
        check(self.lib.zl_block_manager_try_reference(self.handle, ctypes.byref(c)))

    def available(self) -> int:
        return int(self.lib.zl_block_manager_available(self.handle))

    free_blocks = property(available)

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.zl_block_manager_destroy(self.handle)
            self.handle = None


class KVCache:
    """Per-layer paged K/V pools with per-sequence device block tables."""

    def __init__(self, ctx: GpuContext, num_blocks: int, block_size: int, num_layers: int,
                 num_kv_heads: int, head_dim: int, dtype=None):
        import torch
        self.ctx = ctx
        self.lib = ctx.lib
        self.dtype = dtype or torch.float32
        h = ctypes.c_void_p()
        check(self.lib.zl_kv_cache_create(ctx.handle, num_blocks, block_size, num_layers,
                                          num_kv_heads, head_dim, dtype_code(self.dtype),
                                          ctypes.byref(h)))
        self.handle = h
        self.num_blocks, self.block_size, self.num_layers = num_blocks, block_size, num_layers
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim

    def register_seq(self, seq_id: str, max_blocks: int) -> None:
        check(self.lib.zl_kv_cache_register_seq(self.handle, seq_id.encode(), max_blocks))

    def alloc_block(self, seq_id: str, bm: BlockManager) -> BlockHandle:
        out = _capi.zl_block_handle()
        check(self.lib.zl_kv_cache_alloc_block(self.handle, seq_id.encode(), bm.handle, ctypes.byref(out)))
        return BlockHandle(int(out.block_id), int(out.generation))

    def release_seq(self, seq_id: str) -> None:
        check(self.lib.zl_kv_cache_release_seq(self.handle, seq_id.encode()))

    def store_kv(self, layer: int, seq_id: str, k, v, start_token: int, n_tokens: int, stream=None) -> None:
        check(self.lib.zl_kv_cache_store_kv(self.handle, layer, seq_id.encode(), ptr(k), ptr(v),
                                            start_token, n_tokens, self.ctx.stream(stream)))

    def append_kv(self, layer: int, seq_id: str, k, v, stream=None) -> None:
        check(self.lib.zl_kv_cache_append_kv(self.handle, layer, seq_id.encode(), ptr(k), ptr(v),
                                             self.ctx.stream(stream)))

    def cached_tokens(self, seq_id: str) -> int:
        out = ctypes.c_uint64()
        check(self.lib.zl_kv_cache_cached_tokens(self.handle, seq_id.encode(), ctypes.byref(out)))
        return int(out.value)

    def block_table_ptr(self, seq_id: str) -> int:
        return int(self.lib.zl_kv_cache_block_table_ptr(self.handle, seq_id.encode()) or 0)

    def k_pool_ptr(self, layer: int) -> int:
        return int(self.lib.zl_kv_cache_k_pool_ptr(self.handle, layer) or 0)

    def v_pool_ptr(self, layer: int) -> int:
        return int(self.lib.zl_kv_cache_v_pool_ptr(self.handle, layer) or 0)

    def k_pool(self, layer: int):
        """torch view [num_blocks][Hkv][bs][d] of layer `layer`'s K pool."""
        return device_view(self.k_pool_ptr(layer), self._pool_shape(), self.dtype)

    def v_pool(self, layer: int):
        return device_view(self.v_pool_ptr(layer), self._pool_shape(), self.dtype)

    def block_table(self, seq_id: str, max_blocks: int):
        import torch
        return device_view(self.block_table_ptr(seq_id), (max_blocks,), torch.int32)

    def _pool_shape(self):
        return (self.num_blocks, self.num_kv_heads, self.block_size, self.head_dim)

    def pool_elements(self) -> int:
        return self.num_blocks * self.block_size * self.num_kv_heads * self.head_dim

    def __del__(self):
        if getattr(self, "handle", None):
            self.lib.zl_kv_cache_destroy(self.handle)
            self.handle = None
