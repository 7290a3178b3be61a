"""Multi-process host logic on CPU (gloo, world size 2): kv-head-group sharding and the
sequence-split partial/merge protocol, with the oracle standing in for the kernels."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _case(seed=5):
    rng = np.random.default_rng(seed)
    B, H, Hkv, d, bs, nb = 3, 8, 4, 16, 16, 64
    lens = np.array([5, 100, 257], np.int32)
    nblk = (lens + bs - 1) // bs
    perm = rng.permutation(nb).astype(np.int32)
    table = np.full((B, int(nblk.max())), -1, np.int32)
    off = 0
    for b in range(B):
        table[b, : nblk[b]] = perm[off: off + nblk[b]]
        off += nblk[b]
    q = rng.standard_normal((B, H, d)).astype(np.float32)
    kp = rng.standard_normal((nb, Hkv, bs, d)).astype(np.float32)
    vp = rng.standard_normal((nb, Hkv, bs, d)).astype(np.float32)
    return B, H, Hkv, d, bs, nb, lens, table, q, kp, vp


def test_token_split_partitions_each_sequence():
    from zealot_b200.dist import token_split
    lens = np.array([0, 1, 16, 17, 1000, 4096], np.int32)
    for world in (1, 2, 3, 4, 8):
        got = np.zeros_like(lens)
        prev_end = np.zeros_like(lens)
        for r in range(world):
            b, e = token_split(lens, r, world, 16)
            assert np.all(b == prev_end) and np.all(e >= b)
            assert np.all((b % 16 == 0) | (b == lens))
            got += e - b
            prev_end = e
        assert np.array_equal(got, lens)


def test_kv_head_groups():
    from zealot_b200.dist import kv_head_group, query_heads_of
    import zealot_b200 as zb
    assert [kv_head_group(r, 4, 8) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert query_heads_of(2, 4, 32, 8) == (8, 16)
    with pytest.raises(zb.InvalidArgument):
        kv_head_group(0, 3, 8)


def _worker(rank, world, port, mode, q_out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import torch
    from oracle import oracle
    from zealot_b200.dist import kv_head_group, query_heads_of, token_split
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, H, Hkv, d, bs, nb, lens, table, q, kp, vp = _case()
    if mode == "heads":
        lo, hi = kv_head_group(rank, world, Hkv)
        hlo, hhi = query_heads_of(lo, hi, H, Hkv)
        mine = oracle.paged_decode(np.ascontiguousarray(q[:, hlo:hhi]), np.ascontiguousarray(kp[:, lo:hi]),
                                   np.ascontiguousarray(vp[:, lo:hi]), table, lens, hhi - hlo, hi - lo,
                                   d, bs, nb)
        parts = [torch.empty(B, H // world, d) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(mine))
        res = torch.cat(parts, dim=1).numpy()
    else:
        b, e = token_split(lens, rank, world, bs)
        m, l, o = oracle.paged_decode_partial(q, kp, vp, table, b, e, H, Hkv, d, bs, nb)
        gm = [torch.empty(B, H) for _ in range(world)]
        gl = [torch.empty(B, H) for _ in range(world)]
        go = [torch.empty(B, H, d) for _ in range(world)]
        dist.all_gather(gm, torch.from_numpy(m))
        dist.all_gather(gl, torch.from_numpy(l))
        dist.all_gather(go, torch.from_numpy(o))
        res = oracle.merge_partials(torch.stack(gm).numpy(), torch.stack(gl).numpy(),
                                    torch.stack(go).numpy()).reshape(B, H, d)
    dist.destroy_process_group()
    q_out.put((rank, res))


@pytest.mark.parametrize("mode", ["heads", "sequence"])
def test_gloo_two_ranks(oracle, mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, qo)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(qo.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    B, H, Hkv, d, bs, nb, lens, table, q, kp, vp = _case()
    full = oracle.paged_decode(q, kp, vp, table, lens, H, Hkv, d, bs, nb)
    for r in range(2):
        np.testing.assert_allclose(outs[r], full, rtol=1e-5, atol=1e-6)


def _watch_worker(rank, port, scenario, q_out):
    sys.path.insert(0, ROOT)
    import datetime
    import time
    import torch.distributed as dist
    from zealot_b200.dist import PeerWatch
    from zealot_b200.errors import PeerLost
    store = dist.TCPStore("127.0.0.1", port, 2, is_master=(rank == 0),
                          timeout=datetime.timedelta(seconds=30))
    w = PeerWatch(store, rank, 2, timeout_s=1.0)
    res, t0 = [], time.monotonic()
    try:
        for n in range(3):
            if rank == 1 and n == 2:  # rank 1 stops between steps 1 and 2
                if scenario == "leave":
                    w.leave()
                break
            w.step(n)
            res.append(n)
    except PeerLost as e:
        res.append(f"PeerLost: {e}")
    q_out.put((rank, res, time.monotonic() - t0))
    if rank == 0:
        time.sleep(0.5)  # the store lives in rank 0: let rank 1 finish with it


@pytest.mark.parametrize("scenario", ["leave", "crash"])
def test_peer_watch_reports_a_rank_gone_between_steps(scenario):
    """Two ranks (processes) step together; rank 1 stops after step 1, announcing it
    (leave) or not (crash). Rank 0 learns it on the host at step 2 -- at once, or
    after its 1 s deadline -- as PeerLost, before it would launch anything."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_watch_worker, args=(r, port, scenario, qo)) for r in range(2)]
    for p in procs:
        p.start()
    outs = {r: (res, dt) for r, res, dt in (qo.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert outs[1][0] == [0, 1]
    res0 = outs[0][0]
    assert res0[:2] == [0, 1] and len(res0) == 3 and res0[2].startswith("PeerLost: rank 1")
    if scenario == "leave":
        assert "left the job after step 1" in res0[2]
    else:
        assert "did not reach step 2 within 1 s" in res0[2]
