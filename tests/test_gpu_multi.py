"""Two GPUs, one process each: kv-head-group sharding (no collective) and the
sequence split merged with NCCL (zl_nccl_merge), both against the oracle."""
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


def _worker(rank, world, port, q_out):
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
    res = [qo.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, eh, es, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert eh <= 2e-2 and es <= 2e-2, (rank, eh, es)
