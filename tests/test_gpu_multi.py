"""Two GPUs, one process each: kv-head-group sharding (no collective) and the
sequence split merged with NCCL (zl_nccl_merge), both against the oracle; and a
peer that leaves between steps, whose partner's next all-gather is aborted by
the bounded wait (zl_nccl_wait) instead of waiting for good.

NVLS is off in these processes (NCCL_NVLS_ENABLE=0) and no kernel of the
library uses multimem, so a rank that leaves holds no NVLink multicast memory."""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _reap(procs):
    """Joins the rank processes; one that did not finish is killed (its exit tears
    down its CUDA context), so the test never leaves a rank behind."""
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(timeout=30)


def _worker(rank, world, port, q_out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        sys.path.insert(0, ROOT)
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        import zealot_b200 as zb
        from zealot_b200.dist import SequenceSplitDecoder, kv_head_group, query_heads_of, token_split
        from oracle import oracle
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rng = np.random.default_rng(11)
        B, H, Hkv, d, bs, nb = 4, 32, 8, 128, 16, 2048
        lens = np.array([700, 16, 4100, 2500], np.int32)
        nblk = (lens + bs - 1) // bs
        perm = rng.permutation(nb).astype(np.int32)
        table = np.full((B, int(nblk.max())), -1, np.int32)
        off = 0
        for b in range(B):
            table[b, : nblk[b]] = perm[off: off + nblk[b]]
            off += nblk[b]
        q = oracle.round_bf16(rng.standard_normal((B, H, d)).astype(np.float32))
        kp = oracle.round_bf16(rng.standard_normal((nb, Hkv, bs, d)).astype(np.float32))
        vp = oracle.round_bf16(rng.standard_normal((nb, Hkv, bs, d)).astype(np.float32))
        ctx = zb.GpuContext(rank)
        attn = zb.CudaAttention(ctx)
        bf = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(torch.bfloat16)
        tt = torch.from_numpy(table).cuda()
        # 1. kv-head-group sharding: this GPU's pools hold only its kv heads
        lo, hi = kv_head_group(rank, world, Hkv)
        hlo, hhi = query_heads_of(lo, hi, H, Hkv)
        out_h = torch.empty((B, hhi - hlo, d), dtype=torch.bfloat16, device="cuda")
        attn.paged_forward(bf(q[:, hlo:hhi]), bf(kp[:, lo:hi]), bf(vp[:, lo:hi]), tt,
                           torch.from_numpy(lens).cuda(), out_h, B, hhi - hlo, hi - lo, d, bs,
                           table.shape[1], num_blocks=nb)
        ctx.check_status()
        ref = oracle.paged_decode(q, kp, vp, table, lens, H, Hkv, d, bs, nb, num_threads=4)
        err_h = float(np.max(np.abs(out_h.float().cpu().numpy() - ref[:, hlo:hhi])))
        # 2. sequence split: this GPU attends to its block-aligned token range only
        def bcast(x):
            obj = [x]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]
        dec = SequenceSplitDecoder(ctx, rank, world, bcast)
        b, e = token_split(lens, rank, world, bs)
        out_s = torch.empty((B, H, d), dtype=torch.bfloat16, device="cuda")
        dec.decode(bf(q), bf(kp), bf(vp), tt, torch.from_numpy(b).cuda(), torch.from_numpy(e).cuda(),
                   out_s, H, Hkv, d, bs, table.shape[1], num_blocks=nb)
        ctx.check_status()
        err_s = float(np.max(np.abs(out_s.float().cpu().numpy() - ref)))
        dec.close()
        dist.destroy_process_group()
        ctx.close()
        q_out.put((rank, err_h, err_s, None))
    except Exception as ex:  # report, never hang the parent
        q_out.put((rank, None, None, repr(ex)))


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_head_sharding_and_sequence_split():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, qo)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = [qo.get(timeout=300) for _ in procs]
    finally:
        _reap(procs)
    for rank, eh, es, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert eh <= 2e-2 and es <= 2e-2, (rank, eh, es)


def _lost_peer_worker(rank, world, port, q_out):
    """Two good sequence-split steps, then rank 1 leaves between steps (nothing of
    its own in flight) and stays alive without joining step 3. Rank 0's step-3
    all-gather can never finish: zl_nccl_wait must give up after its timeout,
    abort the communicator and report DeviceTimeout; afterwards the context still
    runs single-GPU decode correctly and further merges fail with NcclError."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        sys.path.insert(0, ROOT)
        import time
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        import zealot_b200 as zb
        from zealot_b200.dist import SequenceSplitDecoder, token_split
        from oracle import oracle
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        store = dist.distributed_c10d._get_default_store()
        rng = np.random.default_rng(12)
        B, H, Hkv, d, bs, nb = 3, 16, 4, 128, 16, 1024
        lens = np.array([900, 2000, 33], np.int32)
        nblk = (lens + bs - 1) // bs
        perm = rng.permutation(nb).astype(np.int32)
        table = np.full((B, int(nblk.max())), -1, np.int32)
        off = 0
        for b in range(B):
            table[b, : nblk[b]] = perm[off: off + nblk[b]]
            off += nblk[b]
        q = oracle.round_bf16(rng.standard_normal((B, H, d)).astype(np.float32))
        kp = oracle.round_bf16(rng.standard_normal((nb, Hkv, bs, d)).astype(np.float32))
        vp = oracle.round_bf16(rng.standard_normal((nb, Hkv, bs, d)).astype(np.float32))
        ref = oracle.paged_decode(q, kp, vp, table, lens, H, Hkv, d, bs, nb, num_threads=4)
        ctx = zb.GpuContext(rank)
        bf = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda().to(torch.bfloat16)
        tq, tk, tv, tt = bf(q), bf(kp), bf(vp), torch.from_numpy(table).cuda()

        def bcast(x):
            obj = [x]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]

        dec = SequenceSplitDecoder(ctx, rank, world, bcast, max_rows=B * H, timeout_ms=3000)
        tb, te = (torch.from_numpy(x).cuda() for x in token_split(lens, rank, world, bs))
        out = torch.empty((B, H, d), dtype=torch.bfloat16, device="cuda")
        errs = []
        for _ in range(2):
            dec.decode(tq, tk, tv, tt, tb, te, out, H, Hkv, d, bs, table.shape[1], num_blocks=nb)
            dec.wait()
            ctx.check_status()
            errs.append(float(np.max(np.abs(out.float().cpu().numpy() - ref))))
        dist.barrier()  # both ranks finished step 2; nothing is in flight
        if rank == 1:
            store.wait(["zl/test/rank0_done"], __import__("datetime").timedelta(seconds=120))
            dec.abort()
            ctx.close()
            q_out.put((rank, errs, None, None))
            return
        dec.decode(tq, tk, tv, tt, tb, te, out, H, Hkv, d, bs, table.shape[1], num_blocks=nb)
        t0 = time.monotonic()
        try:
            dec.wait()
            lost = "no error"
        except zb.DeviceTimeout:
            lost = "timeout"
        waited = time.monotonic() - t0
        try:
            dec.decode(tq, tk, tv, tt, tb, te, out, H, Hkv, d, bs, table.shape[1], num_blocks=nb)
            after = "no error"
        except zb.NcclError:
            after = "nccl error"
        # the context still serves single-GPU work
        full = torch.empty((B, H, d), dtype=torch.bfloat16, device="cuda")
        zb.CudaAttention(ctx).paged_forward(tq, tk, tv, tt, torch.from_numpy(lens).cuda(), full, B, H, Hkv,
                                            d, bs, table.shape[1], num_blocks=nb)
        ctx.check_status()
        err_after = float(np.max(np.abs(full.float().cpu().numpy() - ref)))
        store.set("zl/test/rank0_done", "1")
        ctx.close()
        q_out.put((rank, errs, (lost, waited, after, err_after), None))
    except Exception as ex:  # report, never hang the parent
        try:
            dist.distributed_c10d._get_default_store().set("zl/test/rank0_done", "1")
        except Exception:
            pass
        q_out.put((rank, None, None, repr(ex)))


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_lost_peer_aborts_the_collective():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    qo = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lost_peer_worker, args=(r, 2, port, qo)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = sorted(qo.get(timeout=300) for _ in procs)
    finally:
        _reap(procs)
    for rank, errs, info, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert max(errs) <= 2e-2, (rank, errs)
    lost, waited, after, err_after = res[0][2]
    assert lost == "timeout" and 2.5 <= waited <= 30, (lost, waited)
    assert after == "nccl error"
    assert err_after <= 2e-2
