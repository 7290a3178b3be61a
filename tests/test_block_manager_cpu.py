"""The BlockManager through the C ABI, on the CPU.

- A hypothesis state machine against the restated model (oracle.OracleBlockManager):
  the counterpart of the reference's proptest (tests/block_manager_proptest.rs:139-259,
  allocate / free / reference / stale and unknown handles, LIFO ids, generations).
- Several threads allocating and freeing at once (ctypes calls run without the GIL):
  the counterpart of the reference's loom check of the free list
  (src/block_manager.rs:280-550): no id is handed out twice while it is live, and
  every block is free again at the end.
"""
import random
import threading

import pytest
from hypothesis import HealthCheck, settings
from hypothesis import strategies as st
from hypothesis.stateful import RuleBasedStateMachine, initialize, invariant, precondition, rule

import zealot_b200 as zb
from oracle import oracle as O


class BlockManagerModel(RuleBasedStateMachine):
    @initialize(n=st.integers(1, 8))
    def make(self, n):
        self.n = n
        self.bm = zb.BlockManager(n, 16)
        self.ref = O.OracleBlockManager(n, 16)
        self.live = []  # handles held (a referenced block appears once per reference)

    @rule()
    def allocate(self):
        try:
            want = self.ref.try_allocate()
        except MemoryError:
            with pytest.raises(zb.OutOfBlocks):
                self.bm.try_allocate()
            return
        got = self.bm.try_allocate()
        assert (got.block_id, got.generation) == want
        self.live.append(want)

    @precondition(lambda self: self.live)
    @rule(i=st.integers(0, 1 << 16))
    def free(self, i):
        h = self.live.pop(i % len(self.live))
        self.ref.try_free(h)
        self.bm.try_free(zb.BlockHandle(*h))

    @precondition(lambda self: self.live)
    @rule(i=st.integers(0, 1 << 16))
    def reference(self, i):
        h = self.live[i % len(self.live)]
        self.ref.try_reference(h)
        self.bm.try_reference(zb.BlockHandle(*h))
        self.live.append(h)

    @rule(i=st.integers(0, 1 << 16))
    def free_stale(self, i):
        bid = i % self.n
        gen = self.ref.generation[bid] - 1  # a generation already retired
        if gen >= 1:
            with pytest.raises(zb.StaleHandle):
                self.bm.try_free(zb.BlockHandle(bid, gen))

    @rule(i=st.integers(0, 4))
    def free_unknown(self, i):
        with pytest.raises(zb.BlockNotAllocated):
            self.bm.try_free(zb.BlockHandle(self.n + i, 1))

    @invariant()
    def same_available(self):
        if hasattr(self, "bm"):
            assert self.bm.available() == self.ref.available()


TestBlockManagerModel = BlockManagerModel.TestCase
TestBlockManagerModel.settings = settings(max_examples=80, stateful_step_count=60, deadline=None,
                                          suppress_health_check=[HealthCheck.too_slow])


def test_concurrent_allocate_and_free():
    n, threads, ops = 64, 8, 3000
    bm = zb.BlockManager(n, 16)
    held, lock, doubles = set(), threading.Lock(), []

    def worker(seed):
        rng = random.Random(seed)
        mine = []
        for _ in range(ops):
            if mine and (rng.random() < 0.5 or len(mine) >= 12):
                h = mine.pop(rng.randrange(len(mine)))
                with lock:
                    held.discard(h.block_id)  # before the free: the id may be handed out again at once
                bm.try_free(h)
            else:
                try:
                    h = bm.try_allocate()
                except zb.OutOfBlocks:
                    continue
                with lock:
                    if h.block_id in held:
                        doubles.append(h.block_id)
                    held.add(h.block_id)
                mine.append(h)
        for h in mine:
            with lock:
                held.discard(h.block_id)
            bm.try_free(h)

    ts = [threading.Thread(target=worker, args=(s,)) for s in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert doubles == []
    assert bm.available() == n
