"""CPU-side checks of the C ABI: the library loads without a GPU, exports every
symbol include/zealot_attn.h declares, and its host-only parts (BlockManager,
error mapping) behave like the reference."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    hdr = open(os.path.join(ROOT, "include", "zealot_attn.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(zl_[a-z0-9_]+)\s*\(", hdr)))


def test_library_exports_every_declared_symbol():
    from zealot_b200 import _capi
    lib = _capi.load()
    names = _declared()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), f"{n} declared in zealot_attn.h but not exported"
    assert set(names) == set(_capi.SIGNATURES), "ctypes signatures out of sync with the header"


def test_abi_version_and_status_strings():
    from zealot_b200 import _capi
    lib = _capi.load()
    assert lib.zl_abi_version() == 1
    assert lib.zl_status_string(7) == b"out of blocks"


def test_no_device_is_a_loud_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import zealot_b200 as zb
    with pytest.raises(zb.CudaError):
        zb.GpuContext(0)


def test_block_manager_matches_reference_model(oracle):
    """Random allocate / free / reference sequences through the C ABI against the
    restated model (the reference's proptest, tests/block_manager_proptest.rs)."""
    import zealot_b200 as zb
    rng = np.random.default_rng(7)
    for trial in range(20):
        n = int(rng.integers(1, 12))
        bm = zb.BlockManager(n, 16)
        ref = oracle.OracleBlockManager(n, 16)
        live = []
        for _ in range(200):
            op = rng.integers(0, 4)
            if op == 0:
                try:
                    h = ref.try_allocate()
                    got = bm.try_allocate()
                    assert (got.block_id, got.generation) == h
                    live.append(h)
                except MemoryError:
                    with pytest.raises(zb.OutOfBlocks):
                        bm.try_allocate()
            elif op == 1 and live:
                h = live.pop(int(rng.integers(0, len(live))))
                ref.try_free(h)
                bm.try_free(zb.BlockHandle(*h))
            elif op == 2 and live:
                h = live[int(rng.integers(0, len(live)))]
                ref.try_reference(h)
                bm.try_reference(zb.BlockHandle(*h))
                live.append(h)
            elif op == 3:
                # a stale handle: a generation that was already retired
                bid = int(rng.integers(0, n))
                stale = (bid, ref.generation[bid] - 1)
                if stale[1] >= 1:
                    with pytest.raises(zb.StaleHandle):
                        bm.try_free(zb.BlockHandle(*stale))
            assert bm.available() == ref.available()


def test_block_manager_errors():
    import zealot_b200 as zb
    with pytest.raises(zb.InvalidBlockSize):
        zb.BlockManager(4, 0)
    bm = zb.BlockManager(2, 16)
    with pytest.raises(zb.BlockNotAllocated):
        bm.try_free(zb.BlockHandle(5, 1))
    a = bm.try_allocate()
    b = bm.try_allocate()
    assert (a.block_id, b.block_id) == (0, 1)
    with pytest.raises(zb.OutOfBlocks):
        bm.try_allocate()
    bm.try_free(a)
    with pytest.raises(zb.StaleHandle):
        bm.try_free(a)
    assert bm.try_allocate() == zb.BlockHandle(0, 2)
