"""Multi-GPU partitioning of the attention path (one process per GPU).

Two ways to spread the work, matching the north star of the path:

* kv-head-group sharding (no collective): GPU r of N owns kv heads
  [r*Hkv/N, (r+1)*Hkv/N) and their query heads; its pools hold only those
  heads, and every GPU uses the same block ids and tables. Decode and prefill
  outputs are complete heads, so nothing is exchanged.
* sequence split (one sequence's KV spread over GPUs): GPU r attends to a
  contiguous, block-aligned token range of each sequence and produces the
  partial triple (m, l, o); the triples are all-gathered over NVLink with NCCL
  and merged (zl_nccl_merge), since the merge is not a sum.

The reference engine is single-device (`CudaModelRunner::load(id, 0)`,
src/bin/zealot-backend.rs:317); this module has no counterpart there.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np

from .context import GpuContext, GQA_GROUPED, dtype_code, ptr
from .errors import check, InvalidArgument, PeerLost


def kv_head_group(rank: int, world: int, num_kv_heads: int) -> tuple[int, int]:
    """[lo, hi) kv heads owned by `rank`; the kv heads must divide over the GPUs."""
    if world <= 0 or not 0 <= rank < world:
        raise InvalidArgument(f"rank {rank} of {world}")
    if num_kv_heads % world:
        raise InvalidArgument(f"{num_kv_heads} kv heads do not divide over {world} GPUs")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def query_heads_of(kv_lo: int, kv_hi: int, num_heads: int, num_kv_heads: int) -> tuple[int, int]:
    """Query heads [lo, hi) served by kv heads [kv_lo, kv_hi) under the grouped mapping."""
    g = num_heads // num_kv_heads
    return kv_lo * g, kv_hi * g


def token_split(seq_lens, rank: int, world: int, block_size: int):
    """Block-aligned contiguous token range [begin, end) of every sequence for `rank`.

    Each sequence's blocks are dealt out in contiguous runs of equal count (the
    first ranks take one extra block when it does not divide), so a GPU only needs
    the pool blocks of its own range.
    """
    lens = np.asarray(seq_lens, dtype=np.int64)
    nblk = (lens + block_size - 1) // block_size
    base, extra = nblk // world, nblk % world
    b_lo = rank * base + np.minimum(rank, extra)
    b_hi = b_lo + base + (rank < extra)
    begin = np.minimum(b_lo * block_size, lens)
    end = np.minimum(b_hi * block_size, lens)
    return begin.astype(np.int32), end.astype(np.int32)


class PeerWatch:
    """Host-side liveness of the ranks of a multi-GPU job, through the job's
    key-value store (torch.distributed's TCPStore or any object with set / get /
    check). Before every collective step each rank publishes the step it is about
    to run and waits, up to `timeout_s`, until every peer has published it too.
    A peer that left (leave()) or stopped between steps is reported as PeerLost
    before this rank launches anything for the step, so no collective is ever
    left waiting on the GPU for a rank that is gone."""

    LEFT = "left:"  # + the last step the rank reached: peers still pass steps up to it

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "zl/peer/"):
        if world <= 0 or not 0 <= rank < world or timeout_s <= 0:
            raise InvalidArgument(f"rank {rank} of {world}, timeout {timeout_s}")
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix
        self.last = -1

    def _key(self, r: int) -> str:
        return f"{self.prefix}{r}"

    def _read(self, r: int) -> str | None:
        key = self._key(r)
        if not self.store.check([key]):
            return None
        v = self.store.get(key)
        return v.decode() if isinstance(v, (bytes, bytearray)) else str(v)

    def step(self, n: int) -> None:
        """Returns once every peer has reached step n; raises PeerLost otherwise."""
        try:
            self.store.set(self._key(self.rank), str(n))
            self.last = n
            deadline = time.monotonic() + self.timeout_s
            for peer in range(self.world):
                if peer == self.rank:
                    continue
                while True:
                    v = self._read(peer)
                    if v is not None and v.startswith(self.LEFT):
                        gone_after = int(v[len(self.LEFT):])
                        if gone_after >= n:
                            break
                        raise PeerLost(f"rank {peer} left the job after step {gone_after}, before step {n}")
                    if v is not None and int(v) >= n:
                        break
                    if time.monotonic() > deadline:
                        raise PeerLost(f"rank {peer} did not reach step {n} within {self.timeout_s:g} s "
                                       f"(last at step {v})")
                    time.sleep(0.002)
        except PeerLost:
            raise
        except Exception as e:  # the store itself is gone with the rank that hosted it
            raise PeerLost(f"the job's store stopped answering at step {n}: {e}") from e

    def leave(self) -> None:
        """Tells the peers that this rank is gone (their next step() raises at once)."""
        try:
            self.store.set(self._key(self.rank), f"{self.LEFT}{self.last}")
        except Exception:
            pass


class SequenceSplitDecoder:
    """Decode for sequences whose KV is split across GPUs: local partial triples,
    NCCL all-gather over NVLink, merge kernel. One instance per process/GPU."""

    def __init__(self, ctx: GpuContext, rank: int, world: int, broadcast_id, watch: PeerWatch | None = None,
                 max_rows: int = 4096, max_head_dim: int = 128, timeout_ms: int = 10000):
        """`broadcast_id(bytes_or_None) -> bytes` shares rank 0's 128-byte NCCL id
        (e.g. via torch.distributed.broadcast_object_list). With `watch`, every
        decode() first checks that all ranks reached the same step (PeerLost
        otherwise) before it launches the partial decode and the NCCL merge.
        The gather buffer is sized once for steps of up to `max_rows` (sequence,
        head) rows; `timeout_ms` bounds every wait on a collective, after which
        the communicator is aborted (DeviceTimeout) instead of waiting for a
        peer that is gone."""
        self.ctx, self.lib, self.rank, self.world = ctx, ctx.lib, rank, world
        self.watch, self._step = watch, 0
        self._parts = {}
        buf = (ctypes.c_uint8 * 128)()
        if rank == 0:
            check(self.lib.zl_nccl_get_unique_id(buf))
            uid = broadcast_id(bytes(buf))
        else:
            uid = broadcast_id(None)
        ctypes.memmove(buf, uid, 128)
        check(self.lib.zl_nccl_init(ctx.handle, buf, world, rank, max_rows, max_head_dim, timeout_ms))

    def decode(self, q, k_pool, v_pool, block_tables, tok_begin, tok_end, out, num_heads: int,
               num_kv_heads: int, head_dim: int, block_size: int, max_blocks_per_seq: int,
               num_blocks: int | None = None, scale: float = 0.0, gqa_map: int = GQA_GROUPED,
               stream=None) -> None:
        import torch
        if self.watch is not None:
            self.watch.step(self._step)
            self._step += 1
        B = tok_end.numel()
        # the partial triples live as long as the decoder (no allocation per step,
        # and never memory the caching allocator could hand to another stream)
        key = (B, num_heads, head_dim, q.device)
        if key not in self._parts:
            m = torch.empty((B, num_heads), dtype=torch.float32, device=q.device)
            self._parts[key] = (m, torch.empty_like(m),
                                torch.empty((B, num_heads, head_dim), dtype=torch.float32, device=q.device))
        m, l, o = self._parts[key]
        if num_blocks is None:
            num_blocks = k_pool.numel() // (block_size * num_kv_heads * head_dim)
        st = self.ctx.stream(stream)
        check(self.lib.zl_paged_decode_partial(
            self.ctx.handle, ptr(q), ptr(k_pool), ptr(v_pool), ptr(block_tables), ptr(tok_begin),
            ptr(tok_end), ptr(m), ptr(l), ptr(o), B, num_heads, num_kv_heads, head_dim, block_size,
            max_blocks_per_seq, num_blocks, scale, gqa_map, dtype_code(q.dtype), st))
        check(self.lib.zl_nccl_merge(self.ctx.handle, ptr(m), ptr(l), ptr(o), B * num_heads,
                                     head_dim, ptr(out), dtype_code(out.dtype), st))

    def wait(self, timeout_ms: int = 0) -> None:
        """Bounded wait for the last step's all-gather (0: the init timeout). Raises
        DeviceTimeout (and aborts the communicator) when a peer never joined it."""
        check(self.lib.zl_nccl_wait(self.ctx.handle, timeout_ms))

    def abort(self) -> None:
        """Aborts the communicator (e.g. after PeerLost); later decode() calls fail."""
        check(self.lib.zl_nccl_abort(self.ctx.handle))

    def close(self) -> None:
        check(self.lib.zl_nccl_finalize(self.ctx.handle))
        if self.watch is not None:
            self.watch.leave()
