"""bench.py's contract, on the CPU: the reference arm's JSON line (what the driver
runs beside the GPU arm) and the byte model the roofline divides by."""
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "paged_decode_tokens_per_s" and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["warmup"] >= 3 and line["steps"] == 1
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["config"]["global_batch"] == 64


def test_decode_byte_model():
    import bench
    lens, tables, pool = bench.make_lens_tables()
    tables = tables[0]
    assert len(lens) == 64 and lens.min() >= 512 and lens.max() <= 4096
    nblk = (lens.astype(np.int64) + 15) // 16
    # every referenced block id is distinct and inside the pool; -1 after each sequence's blocks
    used = np.concatenate([tables[b, :nblk[b]] for b in range(64)])
    assert len(np.unique(used)) == used.size and used.min() >= 0 and used.max() < pool
    assert all((tables[b, nblk[b]:] == -1).all() for b in range(64))
    # K and V of every token of every kv head, q in + out, table entries and lengths
    want = int(lens.sum()) * 8 * 128 * 2 * 2 + 64 * 32 * 128 * 2 * 2 + int(nblk.sum()) * 4 + 64 * 4
    assert bench.algorithmic_bytes(lens, 8, 32) == want
    # the committed ncu summary of the same launch: traffic within 2 % of the byte model
    traffic = bench.load_traffic("decode_c2_paged_decode_bf16")
    assert traffic is not None and abs(traffic / want - 1) < 0.02


def test_rotated_table_sets_are_disjoint():
    """At N >= 2 the headline rotates over table sets on disjoint pool blocks with the
    same context lengths; the first set is the 1-GPU job's table."""
    import bench
    lens1, t1, _ = bench.make_lens_tables()
    lens, tabs, pool = bench.make_lens_tables(n_sets=bench.ROTATE)
    assert np.array_equal(lens, lens1) and np.array_equal(tabs[0], t1[0])
    nblk = (lens.astype(np.int64) + 15) // 16
    used = [np.concatenate([tabs[s, b, :nblk[b]] for b in range(64)]) for s in range(bench.ROTATE)]
    allb = np.concatenate(used)
    assert len(np.unique(allb)) == allb.size and allb.max() < pool


def test_c5_shape_and_token_split():
    """C5: 8 sequences of 131072 tokens fill the 65536-block pool; the token split
    gives every rank a block-aligned range and the ranges tile each sequence."""
    import bench
    from zealot_b200.dist import token_split
    lens, tabs, pool = bench.make_lens_tables(bench.DECODE_SHAPES["c5"], 1, 0)
    assert (lens == 131072).all() and pool == 65536
    assert np.array_equal(np.sort(tabs[0].reshape(-1)), np.arange(65536))
    for world in (2, 4, 8):
        parts = [token_split(lens, r, world, 16) for r in range(world)]
        assert (parts[0][0] == 0).all() and (parts[-1][1] == lens).all()
        for (b0, e0), (b1, e1) in zip(parts, parts[1:]):
            assert (e0 == b1).all() and (b1 % 16 == 0).all()
