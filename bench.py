"""Benchmark of the Zealot attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: one paged-decode attention step of a
Llama-3-8B layer -- 64 sequences, 32 query / 8 kv heads, head_dim 128, bf16,
context U[512, 4096], block_size 16, block tables drawn from a seeded random
permutation of a 65536-block pool, q/K/V ~ N(0, 1). A step is one
zl_paged_decode launch over every sequence; tokens/s = sequences / step time.

Multi-GPU (torchrun, one process per GPU): the same fixed job, kv-head-group
sharded (strong scaling): rank r owns kv heads [r*8/N, (r+1)*8/N) of all 64
sequences and their query heads; no collective touches the data path. The step
time is the maximum over ranks of CUDA-event time. At N >= 2 a rank's KV per
step is at most 290 MB, so consecutive steps rotate over four sets of block
tables on disjoint pool blocks (same context lengths): no step finds the
previous steps' KV in the 126 MB L2.

The JSON line also carries, at every N (per-rank times and roofline fractions
in each):
  c5                 BASELINE config 5 (8 x 131072 tokens, 64 / 8 heads), its kv
                     heads sharded over the ranks, split-KV inside each GPU;
  seq_split          (N >= 2) the same C5 data split by token range instead:
                     each rank's partial triples (zl_paged_decode_partial) are
                     all-gathered over NVLink and merged (zl_nccl_merge); the
                     merged output is compared with the head-sharded one;
  prefill            C3 varlen causal prefill, heads sharded like the decode;
  reshape_and_cache  the C3 tokens scattered into a paged pool, heads sharded;
plus e2e (the headline through the C ABI with pinned host buffers copied in and
out inside the timed region), sampled clocks and, at N = 1, CPU baselines (the
oracle, a C restatement of the reference CPU path, on one thread, as the
reference runs). `--impl reference` times that oracle alone on all host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B_C2, H, HKV, D, BS, NUM_BLOCKS, MAX_BLOCKS = 64, 32, 8, 128, 16, 65536, 256
B_PER_GPU = B_C2  # the 1-GPU job (kept for the CPU tests of the byte model)
CTX_LO, CTX_HI = 512, 4096
SEED = 2024
ROTATE = 4              # block-table sets rotated at N >= 2
L2_FLUSH_BYTES = 256 << 20

# Decode workloads. C2 (headline): Llama-3-8B layer, the fixed 64-sequence job.
# C5: Llama-3-70B attention, the fixed 8 x 131072 job. Both kv-head sharded.
DECODE_SHAPES = {
    "decode": dict(name="C2", B=64, H=32, HKV=8, ctx=(512, 4096), max_blocks=256, seed=SEED),
    "c5": dict(name="C5", B=8, H=64, HKV=8, ctx=(131072, 131072), max_blocks=8192, seed=SEED + 5),
}
C3 = dict(seqs=16, lo=256, hi=8192, seed=3)


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ workload

def make_lens_tables(shape=None, n_sets: int = 1, pool_blocks: int = NUM_BLOCKS):
    """Context lengths and `n_sets` block tables [n_sets][B][max_blocks] over disjoint
    blocks of one seeded permutation of the pool (identical on every rank)."""
    shape = shape or DECODE_SHAPES["decode"]
    rng = np.random.default_rng(shape["seed"])
    B = shape["B"]
    lo, hi = shape["ctx"]
    lens = rng.integers(lo, hi + 1, size=B).astype(np.int32)
    nblk = (lens + BS - 1) // BS
    pool_blocks = max(pool_blocks, int(nblk.sum()) * n_sets)
    perm = rng.permutation(pool_blocks).astype(np.int32)
    tables = np.full((n_sets, B, shape["max_blocks"]), -1, np.int32)
    off = 0
    for s in range(n_sets):
        for b in range(B):
            tables[s, b, : nblk[b]] = perm[off: off + nblk[b]]
            off += nblk[b]
    return lens, tables, pool_blocks


def algorithmic_bytes(lens, hkv, h, esize=2):
    """Bytes one decode step must move: K and V of every context token of every kv
    head, q in, out, block-table entries and seq_lens."""
    nblk = (lens.astype(np.int64) + BS - 1) // BS
    kv = int(lens.astype(np.int64).sum()) * hkv * D * 2 * esize
    qo = len(lens) * h * D * 2 * esize
    return kv + qo + int(nblk.sum()) * 4 + len(lens) * 4


def c3_lens():
    rng = np.random.default_rng(C3["seed"])
    return rng.integers(C3["lo"], C3["hi"] + 1, size=C3["seqs"]), rng


def prefill_flop(lens, heads):
    return sum(4 * heads * D * int(L) * (int(L) + 1) / 2 for L in lens)


# -------------------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}




# -------------------------------------------------------------- multi-rank

class Ranks:
    """Barrier, max over ranks and per-rank gathers (no-ops on one process)."""

    def __init__(self, dist, rank, world):
        self.dist, self.rank, self.world = dist, rank, world

    def barrier(self):
        import torch
        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize()

    def gather(self, x: float) -> list:
        import torch
        if self.dist is None:
            return [x]
        t = torch.zeros(self.world, device="cuda", dtype=torch.float64)
        t[self.rank] = x
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return [float(v) for v in t.cpu()]

    def max(self, x: float) -> float:
        return max(self.gather(x))


def timed_loop(R, stream, ctx, fn, steps, warmup, between=None):
    """Device time per call of fn(k) on `stream` (CUDA events), the maximum over
    ranks, with a barrier and a synchronize on both sides. Without `between` the
    calls run back to back between two events; with it, every call is bracketed
    by its own events and between() (an L2 flush) runs outside them."""
    import torch
    sh = stream.cuda_stream
    for k in range(warmup):
        fn(k)
    ctx.check_status(sh)
    R.barrier()
    l0 = ctx.launch_count()
    if between is None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(steps):
            fn(k)
        e1.record(stream)
        R.barrier()
        ms = e0.elapsed_time(e1) / steps
    else:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for k in range(steps):
            between()
            ev[k][0].record(stream)
            fn(k)
            ev[k][1].record(stream)
        R.barrier()
        ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    launches = ctx.launch_count() - l0
    ctx.check_status(sh)
    per_rank = R.gather(ms)
    return max(per_rank), per_rank, launches


def roofline(alg_bytes, ms, peak_gbs):
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    return round(gbs, 1), round(gbs / peak_gbs, 4)


# ------------------------------------------------------------------- ours

def run_ours(args, rank, world, local_rank):
    import torch
    import zealot_b200 as zb
    from zealot_b200.context import ptr

    dev = local_rank
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", dev))
    R = Ranks(dist, rank, world)
    peaks = load_peaks()
    shape = DECODE_SHAPES[args.workload]
    Hq, Hk, MAXB = shape["H"], shape["HKV"], shape["max_blocks"]
    assert Hk % world == 0, "kv heads must divide over the GPUs"
    hkv_l, h_l = Hk // world, Hq // world  # this rank's kv-head group
    n_sets = 1 if world == 1 or args.workload == "c5" else ROTATE
    lens, tables, pool_blocks = make_lens_tables(shape, n_sets, args.pool_blocks)
    B = len(lens)
    ctx = zb.GpuContext(dev)
    attn = zb.CudaAttention(ctx)
    stream = torch.cuda.Stream(dev)
    s_handle = stream.cuda_stream
    g = torch.Generator(device="cuda").manual_seed(SEED + rank)
    with torch.cuda.stream(stream):
        kpool = torch.randn((pool_blocks, hkv_l, BS, D), generator=g, device="cuda").to(torch.bfloat16)
        vpool = torch.randn((pool_blocks, hkv_l, BS, D), generator=g, device="cuda").to(torch.bfloat16)
        q = torch.randn((B, h_l, D), generator=g, device="cuda").to(torch.bfloat16)
        out = torch.empty_like(q)
        t_tabs = [torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in tables]
        t_len = torch.from_numpy(lens).cuda()
    stream.synchronize()

    def step(k):
        attn.paged_forward(q, kpool, vpool, t_tabs[k % n_sets], t_len, out, B, h_l, hkv_l, D, BS, MAXB,
                           num_blocks=pool_blocks, stream=s_handle)

    # ---- device-resident timing, clocks sampled over a ~1 s soak and the timed steps
    # The tables and lengths were written once before any timed kernel, so the
    # decode may read them before its dependency wait (ZL_CTX_INPUTS_AHEAD); the
    # e2e loop below uploads them every step and runs with the flag off.
    from zealot_b200.context import CTX_INPUTS_AHEAD
    ctx.set_flags(CTX_INPUTS_AHEAD)
    for k in range(args.warmup):
        step(k)
    ctx.check_status(s_handle)
    clocks = ClockSampler(dev)
    R.barrier()
    clocks.start()
    t_soak = time.perf_counter()
    while not args.lite and time.perf_counter() - t_soak < 1.0:
        for k in range(20):
            step(k)
        stream.synchronize()
    ms_step, ms_ranks, launches = timed_loop(R, stream, ctx, step, args.steps, 0)
    clk = clocks.stop()

    # ---- end to end through the C ABI with pinned host buffers
    # Every step uploads its inputs (q, block tables, seq_lens packed in one
    # pinned buffer) and reads its output back, on copy streams ordered by
    # events. Uploads run AHEAD steps early; before every second kernel (k
    # even) the decode stream waits for the uploads of steps k+1 and k+2, so
    # every kernel's tables and lengths are written before the kernel that
    # precedes it starts (ZL_CTX_INPUTS_AHEAD's contract: the decode may read
    # them before its dependency wait), and half of the kernel-to-kernel
    # boundaries carry no event wait (an event wait between two kernels keeps
    # the second from starting while the first drains; in an engine one table
    # upload serves every layer's decode of the step). The readback of step k
    # overlaps the kernels after it.
    from zealot_b200 import lib
    nbytes = lambda t: t.numel() * t.element_size()
    q_b, tab_b, len_b = nbytes(q), nbytes(t_tabs[0]), nbytes(t_len)
    pack = q_b + tab_b + len_b
    off_tab, off_len = q_b, q_b + tab_b
    AHEAD = 4
    n_buf = max(AHEAD + 2, n_sets)  # steps k .. k + AHEAD in flight, the readback of k - 1
    h_in = [torch.empty(pack, dtype=torch.uint8, pin_memory=True) for _ in range(n_buf)]
    for i, hb in enumerate(h_in):
        hb[:q_b].copy_(q.cpu().view(torch.uint8).reshape(-1))
        hb[off_tab:off_len].copy_(torch.from_numpy(np.ascontiguousarray(tables[i % n_sets])).view(torch.uint8).reshape(-1))
        hb[off_len:].copy_(torch.from_numpy(lens).view(torch.uint8).reshape(-1))
    d_in = [torch.empty(pack, dtype=torch.uint8, device="cuda") for _ in range(n_buf)]
    d_out = [torch.empty_like(out) for _ in range(n_buf)]
    h_out = [torch.empty(out.shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(n_buf)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(n_buf)]
    ev_done = [torch.cuda.Event() for _ in range(n_buf)]
    ev_free = [torch.cuda.Event() for _ in range(n_buf)]
    for e in ev_free:
        e.record(s_out)
    h2d, d2h = pack, nbytes(out)

    def upload(k):
        b = k % n_buf
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_free[b])          # buffer b's previous step is read back
            d_in[b].copy_(h_in[b], non_blocking=True)
            ev_in[b].record(s_in)

    def e2e_step(k):
        upload(k + AHEAD)
        b = k % n_buf
        if k == 0:
            stream.wait_event(ev_in[b])
        if k % 2 == 0:  # the inputs of the next two kernels are written
            stream.wait_event(ev_in[(k + 1) % n_buf])
            stream.wait_event(ev_in[(k + 2) % n_buf])
        base = d_in[b].data_ptr()
        rc = lib.zl_paged_decode(ctx.handle, base, ptr(kpool), ptr(vpool), base + off_tab, base + off_len,
                                 ptr(d_out[b]), B, h_l, hkv_l, D, BS, MAXB, pool_blocks, 0.0, 0, 0, 1,
                                 s_handle)
        assert rc == 0
        ev_done[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[b])
            h_out[b].copy_(d_out[b], non_blocking=True)
            ev_free[b].record(s_out)

    e2e = None
    e2e_launches = 0
    if not args.lite:
        for k in range(AHEAD):
            upload(k)
        gstep = 0  # steps counted across warm-up and timing (buffers and events rotate with it)
        for _ in range(args.warmup):
            e2e_step(gstep)
            gstep += 1
        R.barrier()
        l0 = ctx.launch_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s_in)
        for _ in range(args.steps):
            e2e_step(gstep)
            gstep += 1
        e1.record(s_out)
        e1.synchronize()
        R.barrier()
        e2e_ms = R.max(e0.elapsed_time(e1) / args.steps)
        e2e_launches = ctx.launch_count() - l0
        ctx.check_status(s_handle)
        # the last step's readback equals the device-resident result of the same tables
        last = (gstep - 1) % n_buf
        step(last)
        stream.synchronize()
        assert torch.equal(h_out[last].view(torch.int16), out.cpu().view(torch.int16))
        e2e = {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 5),
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "api": "zl_paged_decode (C ABI) with ZL_CTX_INPUTS_AHEAD; per step one pinned H2D of q + "
                      "block tables + seq_lens (issued four steps ahead; before every second kernel the compute "
                      "stream waits for the next two steps' uploads) and a D2H of out per rank, on copy streams "
                      "that overlap the kernels"}

    # ---- roofline of the decode kernel (one launch per step)
    alg = algorithmic_bytes(lens, hkv_l, h_l)
    achieved, frac = roofline(alg, ms_step, peaks["hbm_gbs"])
    # the committed ncu capture is of the 1-GPU step; other N move different bytes
    traffic = (load_traffic("decode_c2_paged_decode_bf16")
               if world == 1 and args.workload == "decode" else None)
    roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": frac,
            "traffic": traffic, "algorithmic_bytes": alg, "peak_source": peaks["source"],
            "kernel": "paged_decode_bf16_kernel<4,6,false>"}
    per_rank = {"ms": [round(x, 5) for x in ms_ranks],
                "hbm_frac": [roofline(alg, x, peaks["hbm_gbs"])[1] for x in ms_ranks]}
    del kpool, vpool, d_in, d_out
    torch.cuda.empty_cache()

    extra = {}
    if not args.lite and args.workload == "decode":
        extra.update(measure_c5(args, R, ctx, attn, stream, peaks))
        torch.cuda.empty_cache()
        extra.update(measure_c3(args, R, ctx, attn, stream, peaks))
        torch.cuda.empty_cache()
        if world == 1:
            # the engine step (C4) and its steady decode loop on one GPU, each with
            # ~160 GB of weights and paged KV: bounded step counts; a box without the
            # memory (or any failure) records why instead of failing the line
            for key, fn, n in (("c4", measure_c4, 5), ("decode_loop", measure_decode_loop, 10)):
                try:
                    extra[key] = fn(n, 3)
                except (Exception, SystemExit) as ex:
                    extra[key] = {"skipped": f"{type(ex).__name__}: {ex}"[:300]}
                torch.cuda.empty_cache()

    if rank == 0:
        tokens_per_s = B / (ms_step * 1e-3)
        if args.workload == "c5":
            cfg = {"workload": "C5 long-context decode, Llama-3-70B attention shape: 64 q / 8 kv heads, head_dim 128, "
                               "bf16, 8 sequences x 131072 tokens, block_size 16",
                   "global_batch": B, "seq_len": 131072,
                   "parallelism": f"kv-head groups x{world} of the fixed job (rank r: kv heads "
                                  f"[r*{hkv_l}, (r+1)*{hkv_l})), split-KV inside each GPU",
                   "l2": f"inputs larger than L2: {alg / 1e6:.0f} MB of KV read per step per GPU",
                   "launch": "zl_ctx_set_flags(ZL_CTX_INPUTS_AHEAD): device-resident steps read tables written "
                             "once before timing; e2e steps upload theirs four steps ahead"}
        else:
            l2 = (f"inputs larger than L2: {alg / 1e6:.0f} MB of KV read per step per GPU" if n_sets == 1 else
                  f"{alg / 1e6:.0f} MB of KV per step per GPU; steps rotate over {n_sets} block-table sets on "
                  f"disjoint pool blocks ({n_sets * alg / 1e6:.0f} MB per rotation), so no step re-reads the "
                  f"previous steps' KV from L2")
            cfg = {"workload": "C2 paged decode, Llama-3-8B layer shape: 32 q / 8 kv heads, head_dim 128, "
                               "bf16, block_size 16, 65536-block pool per GPU",
                   "global_batch": B, "seq_len": f"U[{CTX_LO},{CTX_HI}]",
                   "parallelism": f"kv-head groups x{world} of the fixed 64-sequence job (rank r: kv heads "
                                  f"[r*{hkv_l}, (r+1)*{hkv_l}) and query heads [r*{h_l}, (r+1)*{h_l}))",
                   "l2": l2,
                   "launch": "zl_ctx_set_flags(ZL_CTX_INPUTS_AHEAD): device-resident steps read tables written "
                             "once before timing; e2e steps upload theirs four steps ahead"}
        line = {
            "metric": "paged_decode_tokens_per_s",
            "value": round(tokens_per_s, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/K/V, random-permutation block tables)",
            "config": cfg,
            "hbm_gbs": achieved,
            "hbm_frac": frac,
            "per_rank": per_rank,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "e2e_gpu_launches": int(e2e_launches),
            "roofline": roof,
            "clocks": clk,
        }
        line.update(extra)
        if world == 1 and not args.no_cpu_baseline and args.workload == "decode":
            line["cpu_baseline"] = cpu_baseline_single(lens, tables[0])
            if "prefill" in line:
                line["prefill"]["cpu_baseline"] = cpu_baseline_prefill()
            if "reshape_and_cache" in line:
                line["reshape_and_cache"]["cpu_baseline"] = cpu_baseline_cache()
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def measure_c5(args, R, ctx, attn, stream, peaks):
    """C5 head-sharded at this N, and (N >= 2) the same data split by token range
    over the ranks and merged with NCCL, with the merged output compared to the
    head-sharded one."""
    import torch
    from zealot_b200.dist import SequenceSplitDecoder, kv_head_group, query_heads_of, token_split
    shape = DECODE_SHAPES["c5"]
    rank, world = R.rank, R.world
    Hq, Hk, MAXB = shape["H"], shape["HKV"], shape["max_blocks"]
    lens, tables, nb = make_lens_tables(shape, 1, 0)
    B = len(lens)
    lo, hi = kv_head_group(rank, world, Hk)
    hlo, hhi = query_heads_of(lo, hi, Hq, Hk)
    sh = stream.cuda_stream
    g = torch.Generator(device="cuda").manual_seed(shape["seed"])  # the same data on every rank
    with torch.cuda.stream(stream):
        kf = torch.randn((nb, Hk, BS, D), generator=g, device="cuda").to(torch.bfloat16)
        vf = torch.randn((nb, Hk, BS, D), generator=g, device="cuda").to(torch.bfloat16)
        qf = torch.randn((B, Hq, D), generator=g, device="cuda").to(torch.bfloat16)
        kc = kf if world == 1 else kf[:, lo:hi].contiguous()
        vc = vf if world == 1 else vf[:, lo:hi].contiguous()
        qc = qf[:, hlo:hhi].contiguous()
        oc = torch.empty_like(qc)
        tt = torch.from_numpy(tables[0]).cuda()
        tl = torch.from_numpy(lens).cuda()
    stream.synchronize()

    def head_step(k):
        attn.paged_forward(qc, kc, vc, tt, tl, oc, B, hhi - hlo, hi - lo, D, BS, MAXB, num_blocks=nb, stream=sh)

    from zealot_b200.context import CTX_INPUTS_AHEAD
    ctx.set_flags(CTX_INPUTS_AHEAD)  # static tables, written before any timed kernel
    ms, ms_r, _ = timed_loop(R, stream, ctx, head_step, args.steps, args.warmup)
    ctx.set_flags(0)
    alg = algorithmic_bytes(lens, hi - lo, hhi - hlo)
    res = {"c5": {"workload": "C5: 8 x 131072 tokens, 64 q / 8 kv heads, d 128, bf16; kv heads sharded over "
                              f"{world} GPU(s) (rank r: kv heads [r*{hi - lo}, (r+1)*{hi - lo})), split-KV inside "
                              "each GPU; inputs larger than L2",
                  "tokens_per_s": round(B / (ms * 1e-3), 1), "ms": round(ms, 5),
                  "hbm_gbs_per_gpu": roofline(alg, ms, peaks["hbm_gbs"])[0],
                  "hbm_frac": roofline(alg, ms, peaks["hbm_gbs"])[1],
                  "per_rank": {"ms": [round(x, 5) for x in ms_r],
                               "hbm_frac": [roofline(alg, x, peaks["hbm_gbs"])[1] for x in ms_r]},
                  "algorithmic_bytes_per_gpu": alg}}
    if world > 1:
        def bcast(x):
            obj = [x]
            R.dist.broadcast_object_list(obj, src=0)
            return obj[0]

        dec = SequenceSplitDecoder(ctx, rank, world, bcast, max_rows=B * Hq, max_head_dim=D, timeout_ms=20000)
        tb, te = token_split(lens, rank, world, BS)
        t_tb, t_te = torch.from_numpy(tb).cuda(), torch.from_numpy(te).cuda()
        os_ = torch.empty((B, Hq, D), dtype=torch.bfloat16, device="cuda")
        m = torch.empty((B, Hq), dtype=torch.float32, device="cuda")
        l = torch.empty_like(m)
        o = torch.empty((B, Hq, D), dtype=torch.float32, device="cuda")

        def partial(k):
            attn.paged_forward_partial(qf, kf, vf, tt, t_tb, t_te, m, l, o, B, Hq, Hk, D, BS, MAXB,
                                       num_blocks=nb, stream=sh)

        def split_step(k):
            dec.decode(qf, kf, vf, tt, t_tb, t_te, os_, Hq, Hk, D, BS, MAXB, num_blocks=nb, stream=sh)

        ms_s, ms_sr, _ = timed_loop(R, stream, ctx, split_step, args.steps, args.warmup)
        dec.wait()
        ms_p, ms_pr, _ = timed_loop(R, stream, ctx, partial, args.steps, args.warmup)
        split_step(0)
        dec.wait()
        ctx.check_status(sh)
        diff = float((os_[:, hlo:hhi].float() - oc.float()).abs().max().item())
        diff = R.max(diff)
        dec.close()
        rng_tokens = (te.astype(np.int64) - tb).sum()
        alg_s = int(rng_tokens) * Hk * D * 2 * 2 + B * Hq * D * 2 + int(((te + BS - 1) // BS - tb // BS).sum()) * 4
        gathered = world * B * Hq * (2 + D) * 4
        res["seq_split"] = {
            "workload": f"C5 data, each sequence's 131072 tokens split into {world} block-aligned ranges (rank r: "
                        "tokens [r*L/N, (r+1)*L/N)) over all 64 heads: zl_paged_decode_partial on the local "
                        "range, then zl_nccl_merge (NCCL all-gather of the (m, l, o) triples over NVLink into "
                        "local HBM + one merge kernel)",
            "tokens_per_s": round(B / (ms_s * 1e-3), 1), "ms": round(ms_s, 5),
            "partial_kernel_ms": round(ms_p, 5), "allgather_and_merge_ms": round(ms_s - ms_p, 5),
            "hbm_frac_partial_kernel": roofline(alg_s, ms_p, peaks["hbm_gbs"])[1],
            "gathered_bytes_per_rank": gathered,
            "max_abs_diff_vs_head_sharded": diff, "tolerance": 2e-2, "parity_ok": diff <= 2e-2,
            "per_rank": {"ms": [round(x, 5) for x in ms_sr], "partial_ms": [round(x, 5) for x in ms_pr]}}
    del kf, vf, kc, vc
    return res


def measure_c3(args, R, ctx, attn, stream, peaks):
    """C3 prefill and reshape_and_cache with this rank's heads; an L2 flush (a
    256 MB write) runs between timed launches, outside the events."""
    import torch
    rank, world = R.rank, R.world
    h, hkv = H // world, HKV // world
    lens, rng = c3_lens()
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    sh = stream.cuda_stream
    g = torch.Generator(device="cuda").manual_seed(C3["seed"] + rank)
    with torch.cuda.stream(stream):
        q = torch.randn((T, h, D), generator=g, device="cuda").to(torch.bfloat16)
        k = torch.randn((T, hkv, D), generator=g, device="cuda").to(torch.bfloat16)
        v = torch.randn((T, hkv, D), generator=g, device="cuda").to(torch.bfloat16)
        o = torch.empty_like(q)
        tcu = torch.from_numpy(cu).cuda()
        flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    stream.synchronize()

    def between():
        with torch.cuda.stream(stream):
            flush.fill_(1.0)

    def pre(i):
        attn.forward_gpu(q, k, v, tcu, o, h, hkv, D, int(lens.max()), causal=True, stream=sh)

    n = max(5, min(args.steps, 20))
    ms, ms_r, _ = timed_loop(R, stream, ctx, pre, n, 3, between)
    flop_rank = prefill_flop(lens, h)
    peak = peaks["bf16_tflops"]
    tf_r = [flop_rank / (x * 1e-3) / 1e12 for x in ms_r]
    res = {"prefill": {"workload": f"C3 varlen causal prefill: 16 seqs, L U[256,8192] (T = {T}), 32/8 heads sharded "
                                   f"over {world} GPU(s) ({h}/{hkv} per GPU), d 128, bf16; L2 flushed between launches",
                       "ms": round(ms, 4), "tflops": round(world * flop_rank / (ms * 1e-3) / 1e12, 2),
                       "tflops_per_gpu": round(min(tf_r), 2), "peak_tflops": peak,
                       "frac": round(min(tf_r) / peak, 4), "flop": world * flop_rank,
                       "per_rank": {"ms": [round(x, 4) for x in ms_r], "frac": [round(x / peak, 4) for x in tf_r]},
                       "kernel": "prefill_tc_kernel (tcgen05.mma kind::f16, TMEM accumulators, TMA)"}}
    # reshape_and_cache of the same tokens into a pool via a random slot mapping
    nb = (T + BS - 1) // BS + 64
    with torch.cuda.stream(stream):
        pk = torch.empty((nb, hkv, BS, D), dtype=torch.bfloat16, device="cuda")
        pv = torch.empty_like(pk)
        slots = torch.from_numpy(rng.permutation(nb * BS)[:T].astype(np.int64)).cuda()
    stream.synchronize()

    def cache(i):
        attn.reshape_and_cache(k, v, pk, pv, slots, hkv, D, BS, nb, stream=sh)

    ms, ms_r, _ = timed_loop(R, stream, ctx, cache, n, 3, between)
    byts = 2 * (T * hkv * D * 2) * 2 + 8 * T
    res["reshape_and_cache"] = {
        "workload": f"C3 tokens ({T}) x {hkv} kv heads per GPU x 128 bf16, random slots; L2 flushed between launches",
        "ms": round(ms, 4), "gbs_per_gpu": roofline(byts, ms, peaks["hbm_gbs"])[0],
        "frac": roofline(byts, ms, peaks["hbm_gbs"])[1], "bytes_per_gpu": byts,
        "per_rank": {"ms": [round(x, 4) for x in ms_r]}}
    del q, k, v, o, pk, pv, flush
    return res


def run_side_only(args):
    """--workload prefill|cache: one side kernel on its C3 workload, own JSON line."""
    import torch
    import zealot_b200 as zb
    torch.cuda.set_device(0)
    ctx = zb.GpuContext(0)
    attn = zb.CudaAttention(ctx)
    stream = torch.cuda.Stream(0)
    R = Ranks(None, 0, 1)
    res = measure_c3(args, R, ctx, attn, stream, load_peaks())
    key = "prefill" if args.workload == "prefill" else "reshape_and_cache"
    r = res[key]
    line = {"metric": "prefill_tflops" if key == "prefill" else "reshape_and_cache_gbs",
            "value": r["tflops"] if key == "prefill" else r["gbs_per_gpu"],
            "unit": "TFLOP/s" if key == "prefill" else "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms"], "higher_is_better": True, "dtype": "bf16",
            "config": {"workload": r["workload"]}, "detail": r}
    print(json.dumps(line), flush=True)
    ctx.close()


C4 = dict(prefill_chunks=8, chunk_len=512, decode_seqs=248, ctx=(1024, 8192), seed=404)


def run_c4(args):
    """--workload c4: the engine-step line (measure_c4)."""
    line = measure_c4(args.steps, args.warmup)
    print(json.dumps(line), flush=True)


def measure_c4(steps, warmup):
    """One engine step of a Mistral-7B-shaped decoder (32 layers,
    d_model 4096, 32/8 heads, d 128, intermediate 14336, vocab 32000, random bf16
    weights): 8 prefill chunks x 512 tokens + 248 decode sequences with context
    U{1024..8192}, batched into one zl_decoder_step. tokens/s = rows per step / step
    time. Inputs (14.5 GB of weights, ~147 GB of KV) are far larger than L2."""
    import torch
    import zealot_b200 as zb
    from zealot_b200.decoder import Decoder, DecoderConfig, StepBatch, random_weights
    torch.cuda.set_device(0)
    cfg = DecoderConfig.mistral_7b()
    rng = np.random.default_rng(C4["seed"])
    dlens = rng.integers(C4["ctx"][0], C4["ctx"][1] + 1, size=C4["decode_seqs"]).astype(np.int32)
    P = C4["prefill_chunks"] * C4["chunk_len"]
    nblk_dec = (dlens + BS - 1) // BS
    nblk = int(nblk_dec.sum()) + C4["prefill_chunks"] * (C4["chunk_len"] // BS)
    pool_bytes = nblk * cfg.num_kv_heads * BS * cfg.head_dim * 2
    weight_bytes = 2 * (cfg.num_layers * sum(int(np.prod(s)) for s in cfg.layer_shapes().values())
                        + 2 * cfg.vocab * cfg.hidden + cfg.hidden)
    need = 2 * cfg.num_layers * pool_bytes + weight_bytes + (4 << 30)
    free, _ = torch.cuda.mem_get_info(0)
    if free < need:
        raise RuntimeError(f"c4 needs {need / 1e9:.1f} GB of device memory, {free / 1e9:.1f} GB free")
    perm = rng.permutation(nblk).astype(np.int32)
    mb = int(nblk_dec.max())
    dtab = np.full((len(dlens), mb), -1, np.int32)
    off = 0
    for i, n in enumerate(nblk_dec):
        dtab[i, :n] = perm[off: off + n]
        off += n
    ptabs = []
    for c in range(C4["prefill_chunks"]):
        n = C4["chunk_len"] // BS
        ptabs.append(list(perm[off: off + n]))
        off += n
    chunks = [rng.integers(0, cfg.vocab, C4["chunk_len"]) for _ in range(C4["prefill_chunks"])]
    dtoks = rng.integers(0, cfg.vocab, len(dlens))
    batch = StepBatch.build(chunks, dtoks, dtab, dlens, ptabs, BS)
    T = P + len(dlens)
    log(f"c4: building weights ({weight_bytes / 1e9:.1f} GB) and pools "
        f"({2 * cfg.num_layers * pool_bytes / 1e9:.1f} GB)")
    w = random_weights(cfg, seed=C4["seed"])
    g = torch.Generator(device="cuda").manual_seed(C4["seed"])
    shape = (nblk, cfg.num_kv_heads, BS, cfg.head_dim)
    kps = [torch.randn(shape, generator=g, device="cuda", dtype=torch.bfloat16)
           for _ in range(cfg.num_layers)]
    vps = [torch.randn(shape, generator=g, device="cuda", dtype=torch.bfloat16)
           for _ in range(cfg.num_layers)]
    ctx = zb.GpuContext(0)
    dec = Decoder(ctx, cfg, w)
    stream = torch.cuda.Stream(0)
    sh = stream.cuda_stream
    logits = torch.empty((batch.num_last, cfg.vocab), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step():
        dec.step(batch, kps, vps, BS, logits=logits, stream=sh)

    for _ in range(warmup):
        step()
    ctx.check_status(sh)
    clocks = ClockSampler(0)
    clocks.start()
    launches0 = ctx.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    e1.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    launches = ctx.launch_count() - launches0
    ctx.check_status(sh)

    # parts of the step timed alone: the attention kernels over all layers
    attn = zb.CudaAttention(ctx)
    Hq, Hk, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    q = torch.randn((T, Hq, d), device="cuda", dtype=torch.bfloat16)
    kv = torch.randn((P, Hk, d), device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(q)

    def time_it(fn, n=3):
        for _ in range(2):
            fn()
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / n

    def dec_all():
        for l in range(cfg.num_layers):
            attn.paged_forward(q[P:], kps[l], vps[l], batch.block_tables, batch.seq_lens, o[P:],
                               len(dlens), Hq, Hk, d, BS, mb, stream=sh)

    def pre_all():
        for l in range(cfg.num_layers):
            attn.forward_gpu(q[:P], kv, kv, batch.cu_prefill, o[:P], Hq, Hk, d, C4["chunk_len"],
                             causal=True, stream=sh)

    ms_dec, ms_pre = time_it(dec_all), time_it(pre_all)
    ctx.check_status(sh)

    # sampling the step's rows on the device vs copying the logits to the host
    from zealot_b200.sampling import GpuSampler, SamplingParams
    sampler = GpuSampler(ctx)
    kinds = [SamplingParams(temperature=0.0), SamplingParams(temperature=0.7, top_k=50, top_p=0.9),
             SamplingParams(top_p=0.95, repetition_penalty=1.1)]
    sparams = [kinds[i % 3] for i in range(batch.num_last)]
    prev = [list(rng.integers(0, cfg.vocab, 64)) for _ in range(batch.num_last)]
    unif = torch.from_numpy(rng.random(batch.num_last).astype(np.float32)).cuda()
    t0 = time.perf_counter()
    sbatch = sampler.prepare(batch.num_last, cfg.vocab, sparams, prev)
    torch.cuda.synchronize()
    ms_prep = (time.perf_counter() - t0) * 1e3
    sout = sampler.launch(sbatch, logits, unif, stream=sh)
    ms_sample = time_it(lambda: sampler.launch(sbatch, logits, unif, out=sout, stream=sh), n=10)
    # the same rows on the host: the restated reference sampler, a bounded sample of rows
    from oracle import oracle as _oracle
    host_logits_np = logits.cpu().numpy()
    ur = unif.cpu().numpy()
    n_cpu = 24
    t0 = time.perf_counter()
    for i in range(n_cpu):
        p = sparams[i]
        _oracle.sample(host_logits_np[i], prev=prev[i], temperature=p.temperature, top_k=p.top_k,
                       top_p=p.top_p, repetition_penalty=p.repetition_penalty, r=float(ur[i]))
    ms_cpu_row = (time.perf_counter() - t0) * 1e3 / n_cpu
    host_logits = torch.empty(logits.shape, dtype=torch.float32, pin_memory=True)

    def d2h():
        with torch.cuda.stream(stream):
            host_logits.copy_(logits, non_blocking=True)

    ms_d2h = time_it(d2h, n=10)
    ctx.check_status(sh)
    peaks = load_peaks()
    params_layer = sum(int(np.prod(s)) for k, s in cfg.layer_shapes().items() if len(s) == 2)
    gemm_flop = 2.0 * T * params_layer * cfg.num_layers + 2.0 * batch.num_last * cfg.vocab * cfg.hidden
    pre_flop = cfg.num_layers * C4["prefill_chunks"] * 4 * Hq * d * C4["chunk_len"] * (C4["chunk_len"] + 1) / 2
    kv_bytes = cfg.num_layers * float(dlens.astype(np.int64).sum()) * Hk * d * 2 * 2
    # A step of ~70 ms of back-to-back GEMMs runs under the power cap: its tensor
    # roofline is the sustained bf16 figure; the burst one is reported beside it.
    kv_ms = 1e3 * kv_bytes / (peaks["hbm_gbs"] * 1e9)
    ideal_ms = 1e3 * (gemm_flop + pre_flop) / (peaks["bf16_tflops_sustained"] * 1e12) + kv_ms
    ideal_burst_ms = 1e3 * (gemm_flop + pre_flop) / (peaks["bf16_tflops"] * 1e12) + kv_ms
    line = {"metric": "engine_step_tokens_per_s", "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s",
            "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random bf16 weights and KV)",
            "config": {"workload": "C4 engine step, Mistral-7B shape (32 layers, d_model 4096, 32/8 heads, "
                                   "d 128, intermediate 14336, vocab 32000): 8 prefill chunks x 512 + "
                                   "248 decode seqs, ctx U[1024,8192]; inputs larger than L2",
                       "rows_per_step": T, "kv_tokens": int(dlens.sum())},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor+hbm", "ideal_ms": round(ideal_ms, 3), "frac": round(ideal_ms / ms, 4),
                         "tensor_peak": "bf16_tflops_sustained",
                         "ideal_ms_at_burst_peak": round(ideal_burst_ms, 3),
                         "frac_of_burst": round(ideal_burst_ms / ms, 4),
                         "gemm_tflop": round(gemm_flop / 1e12, 3), "prefill_attn_tflop": round(pre_flop / 1e12, 3),
                         "decode_kv_gb": round(kv_bytes / 1e9, 2), "peaks": peaks},
            "parts_ms": {"paged_decode_32_layers": round(ms_dec, 3), "prefill_32_layers": round(ms_pre, 3),
                         "rest (GEMMs, norms, cache writes)": round(ms - ms_dec - ms_pre, 3),
                         "gemm_tflops_if_rest": round(gemm_flop / ((ms - ms_dec - ms_pre) * 1e-3) / 1e12, 1)},
            "sampling": {"rows": batch.num_last, "vocab": cfg.vocab,
                         "params": "greedy / t0.7 top-k 50 top-p 0.9 / top-p 0.95 + repetition 1.1, 64 previous ids",
                         "zl_sample_kernel_ms": round(ms_sample, 4),
                         "host_prepare_ms": round(ms_prep, 3),
                         "logits_d2h_ms": round(ms_d2h, 4),
                         "cpu_reference_ms": round(ms_cpu_row * batch.num_last, 2),
                         "note": "kernel = one zl_sample launch over device-resident inputs (CUDA events); "
                                 "host_prepare = packing params / penalty lists and their H2D (wall clock, once "
                                 "per step); cpu_reference = the restated reference sampler (oracle, 1 thread) "
                                 f"timed on {n_cpu} rows and scaled to all rows, plus the logits D2H it needs"},
            "clocks": clk}
    ctx.close()
    return line


def run_decode_loop(args):
    """--workload decode-loop: the decode-loop line (measure_decode_loop)."""
    line = measure_decode_loop(args.steps, args.warmup)
    print(json.dumps(line), flush=True)


def measure_decode_loop(steps, warmup):
    """Steady-state decode steps of the Mistral-7B-shaped
    decoder through the device-resident loop (zl_decode_graph), replayed as a
    CUDA graph and, for comparison, as the same launches issued eagerly.
    Rows 32 and 248 (contexts U{1024..8192}, random bf16 KV and weights); a step
    = block bookkeeping on the host, staging copy, 32 layers, sampling, token
    ids back to pinned host memory. tokens/s = active rows / step time."""
    import torch
    import zealot_b200 as zb
    from zealot_b200.decoder import Decoder, DecoderConfig, DecodeGraph, random_weights
    from zealot_b200.sampling import SamplingParams as SP
    torch.cuda.set_device(0)
    cfg = DecoderConfig.mistral_7b()
    rng = np.random.default_rng(505)
    R = 248
    warm = warmup
    lens = rng.integers(1024, 8193, size=R).astype(np.int32)
    extra = (steps + warm) * 2 + 4  # every row runs all steps of both modes and both sizes
    mb = int((lens.max() + extra * 2 + BS - 1) // BS) + 1
    nblk = int(((lens + BS - 1) // BS).sum()) + R * (extra * 2 // BS + 2)
    w = random_weights(cfg, seed=505)
    g = torch.Generator(device="cuda").manual_seed(505)
    shape = (nblk, cfg.num_kv_heads, BS, cfg.head_dim)
    kps = [torch.randn(shape, generator=g, device="cuda", dtype=torch.bfloat16) for _ in range(cfg.num_layers)]
    vps = [torch.randn(shape, generator=g, device="cuda", dtype=torch.bfloat16) for _ in range(cfg.num_layers)]
    ctx = zb.GpuContext(0)
    dec = Decoder(ctx, cfg, w)
    stream = torch.cuda.Stream(0)
    kinds = [SP(temperature=0.0), SP(temperature=0.7, top_k=50, top_p=0.9), SP(top_p=0.95, repetition_penalty=1.1)]
    res = {}
    for rows in (32, R):
        for use_graph in (True, False):
            perm = list(rng.permutation(nblk))
            dg = DecodeGraph(dec, kps, vps, BS, rows=rows, max_blocks_per_seq=mb, use_graph=use_graph)
            for r in range(rows):
                nb = (int(lens[r]) + BS - 1) // BS
                dg.set_row(r, [int(perm.pop()) for _ in range(nb)], int(lens[r]),
                           int(rng.integers(0, cfg.vocab)), kinds[r % 3],
                           history=list(rng.integers(0, cfg.vocab, 32)))

            def one():
                dg.step({r: int(perm.pop()) for r in dg.rows_needing_block()},
                        rng.random(rows).astype(np.float32), stream=stream)

            for _ in range(warm):
                one()
            dg.tokens()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            e0.record(stream)
            for _ in range(steps):
                one()
            e1.record(stream)
            host_s = (time.perf_counter() - t0) / steps
            e1.synchronize()
            ms = e0.elapsed_time(e1) / steps
            dg.tokens()
            ctx.check_status(stream.cuda_stream)
            key = f"rows{rows}_{'graph' if use_graph else 'eager'}"
            res[key] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(rows / (ms * 1e-3), 1),
                        "host_us_per_step": round(host_s * 1e6, 1)}
            if use_graph:
                res[key]["graph_kernel_nodes"] = dg.num_kernels
            dg.close()
    line = {"metric": "decode_loop_tokens_per_s", "value": res[f"rows{R}_graph"]["tokens_per_s"],
            "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": warm,
            "ms_per_step": res[f"rows{R}_graph"]["ms_per_step"], "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (seeded random bf16 weights and KV)",
            "config": {"workload": "steady-state decode of a Mistral-7B-shaped decoder (32 layers) through "
                                   "zl_decode_graph: rows with contexts U[1024,8192], greedy / top-k+top-p / "
                                   "top-p+repetition sampling; inputs larger than L2"},
            "modes": res}
    ctx.close()
    return line


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 1400.0)),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(name):
    """DRAM bytes per launch (dram__bytes_read.sum + write.sum) from the committed ncu
    summary of the same kernel on the same batch (profiles/<name>.md)."""
    p = os.path.join(ROOT, "profiles", f"{name}.md")
    if os.path.exists(p):
        for line in open(p):
            if line.startswith("dram_bytes_per_launch:"):
                return int(line.split(":")[1])
    return None


# ------------------------------------------------------------- CPU baselines

def _oracle_inputs(lens, tables, hkv, h, n_seqs):
    """fp32 host copies of a sample of the workload, pool compacted to the referenced blocks."""
    from oracle import oracle
    rng = np.random.default_rng(SEED + 99)
    lens = lens[:n_seqs]
    tables = tables[:n_seqs]
    nblk = (lens + BS - 1) // BS
    used = np.concatenate([tables[b, : nblk[b]] for b in range(n_seqs)])
    remap = {int(x): i for i, x in enumerate(used)}
    t2 = np.full_like(tables, -1)
    for b in range(n_seqs):
        t2[b, : nblk[b]] = [remap[int(x)] for x in tables[b, : nblk[b]]]
    kp = oracle.round_bf16(rng.standard_normal((used.size, hkv, BS, D)).astype(np.float32))
    vp = oracle.round_bf16(rng.standard_normal((used.size, hkv, BS, D)).astype(np.float32))
    q = oracle.round_bf16(rng.standard_normal((n_seqs, h, D)).astype(np.float32))
    return q, kp, vp, t2, lens


def cpu_baseline_prefill():
    """The oracle's causal prefill (CpuAttention rows, src/attention/mod.rs:31-103),
    one thread, on a seeded subset of C3 (sequences 1 and 2, one query head and its
    kv head), scaled to the whole C3 job by exact FLOP: extrapolated."""
    from oracle import oracle
    lens, _ = c3_lens()
    sub = [int(lens[1]), int(lens[2])]
    rng = np.random.default_rng(C3["seed"] + 7)
    T = sum(sub)
    cu = np.array([0, sub[0], T], np.int32)
    q, k, v = (oracle.round_bf16(rng.standard_normal((T, 1, D)).astype(np.float32)) for _ in range(3))
    t0, reps = time.perf_counter(), 0
    while True:
        oracle.prefill_varlen(q, k, v, cu, 1, 1, D, causal=True, num_threads=1)
        reps += 1
        if time.perf_counter() - t0 > 3.0:
            break
    dt = (time.perf_counter() - t0) / reps
    tflops = prefill_flop(sub, 1) / dt / 1e12
    job_s = prefill_flop(lens, H) / (tflops * 1e12)
    return {"value": round(tflops, 6), "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "job_s_extrapolated": round(job_s, 1),
            "sample": f"C3 sequences 1-2 (L = {sub[0]}, {sub[1]}), 1 head, {reps} repetitions of {dt:.2f} s; "
                      "scaled to the 16-sequence, 32-head job by exact FLOP (extrapolated); oracle/zl_oracle.c"}


def cpu_baseline_cache():
    """The oracle's store_kv offset arithmetic (src/kv_cache.rs:212-276), one thread,
    on 8192 of the C3 tokens with all 8 kv heads; GB/s of the same byte model."""
    from oracle import oracle
    rng = np.random.default_rng(C3["seed"] + 8)
    T = 8192
    nb = T // BS + 64
    k = oracle.round_bf16(rng.standard_normal((T, HKV, D)).astype(np.float32))
    v = oracle.round_bf16(rng.standard_normal((T, HKV, D)).astype(np.float32))
    kp = np.zeros((nb, HKV, BS, D), np.float32)
    vp = np.zeros_like(kp)
    slots = rng.permutation(nb * BS)[:T].astype(np.int64)
    t0, reps = time.perf_counter(), 0
    while True:
        oracle.reshape_and_cache(kp, vp, k, v, slots, HKV, D, BS, nb)
        reps += 1
        if time.perf_counter() - t0 > 2.0:
            break
    dt = (time.perf_counter() - t0) / reps
    byts = 2 * (T * HKV * D * 2) * 2 + 8 * T  # the GPU's bf16 byte model for the same tokens
    return {"value": round(byts / dt / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{T} C3 tokens x 8 kv heads, {reps} repetitions of {dt * 1e3:.1f} ms; byte model of the bf16 "
                      "GPU call (the oracle copies fp32 rows); oracle/zl_oracle.c"}


def cpu_baseline_single(lens, tables):
    """The oracle port, single-threaded like the reference CpuAttention, on a sample of
    the C2 step (the first 16 of 64 sequences, all heads); scaled to tokens/s."""
    from oracle import oracle
    n = 16
    q, kp, vp, t2, l2 = _oracle_inputs(lens, tables, HKV, H, n)
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.paged_decode(q, kp, vp, t2, l2, H, HKV, D, BS, kp.shape[0], num_threads=1)
        reps += 1
        if time.perf_counter() - t0 > 10.0:
            break
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(n / dt, 2), "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"{n} of the 64 C2 sequences (all 32 heads, contexts as in the GPU run), "
                      f"{reps} repetitions, {dt:.2f} s each; oracle/zl_oracle.c single thread"}


def run_reference(args, rank, world):
    """The reference CPU attention (oracle port) on all host cores, same metric/config."""
    if rank != 0:
        return
    from oracle import oracle
    cores = os.cpu_count() or 1
    lens, tables, _ = make_lens_tables()
    tables = tables[0]
    B = len(lens)
    hkv, h = HKV, H  # the whole job's heads: the CPU does every shard's work
    n = min(B, 64)
    q, kp, vp, t2, l2 = _oracle_inputs(lens, tables, hkv, h, n)
    for _ in range(args.warmup):
        oracle.paged_decode(q, kp, vp, t2, l2, h, hkv, D, BS, kp.shape[0], num_threads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.paged_decode(q, kp, vp, t2, l2, h, hkv, D, BS, kp.shape[0], num_threads=cores)
    dt = (time.perf_counter() - t0) / args.steps
    val = n / dt
    line = {"impl": "reference", "metric": "paged_decode_tokens_per_s", "value": round(val, 2),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) bf16-rounded q/K/V, U[512,4096] contexts)",
            "config": {"workload": "C2 paged decode, Llama-3-8B layer shape (CPU reference path)",
                       "global_batch": B, "sample_seqs_per_step": n, "seq_len": f"U[{CTX_LO},{CTX_HI}]",
                       "parallelism": f"{cores} host threads (OpenMP over (seq, head))"},
            "cpu_baseline": {"value": round(val, 2), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{n} sequences x 32 heads per step of the {B}-sequence job"},
            "e2e": {"value": round(val, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["decode", "c5", "prefill", "cache", "c4", "decode-loop"],
                    default="decode",
                    help="decode (C2, the headline), c5 (long-context decode), a single side kernel "
                         "on its C3 workload, c4 (a full Mistral-7B-shaped engine step, 1 GPU) or "
                         "decode-loop (its steady-state decode through the CUDA-graph loop, 1 GPU)")
    ap.add_argument("--lite", action="store_true",
                    help="only warm-up + timed steps of the kernel (no clock soak, e2e, side runs or "
                         "CPU baseline): the form used under ncu")
    ap.add_argument("--pool-blocks", type=int, default=NUM_BLOCKS,
                    help="KV pool size in blocks per GPU; 0 = just the blocks the batch references")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    # torchrun sets WORLD_SIZE; a plain `python bench.py --gpus N` without it is one process.
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world:
        log(f"note: --gpus {args.gpus} but WORLD_SIZE={world}; running {world} rank(s)")
    if args.lite:
        args.no_cpu_baseline = True
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload in ("prefill", "cache"):
        run_side_only(args)
        return
    if args.workload in ("c4", "decode-loop"):
        if world > 1:
            raise SystemExit(f"--workload {args.workload} runs on one GPU")
        (run_c4 if args.workload == "c4" else run_decode_loop)(args)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
