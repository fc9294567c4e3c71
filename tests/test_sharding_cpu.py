"""Row sharding of the multi-GPU benchmark, on the CPU with two gloo ranks.

bench.py splits rows into contiguous shards, one per rank (cfg1-cfg4 split the
config's rows N ways; cfg5 gives every rank a 50M / 8 slice), each rank
regenerating its own slice from the seeds (synth.make_data's per-chunk seed
spawns), with torch.distributed (gloo) only for barriers and the max over
ranks.  These tests check that the shards of N ranks are disjoint and cover the
whole workload, that a rank's regenerated slice equals the same rows of the full
matrix, and -- with two real gloo processes -- that the per-rank predictions
(the oracle stands in for the GPU here) assemble into the single-process
result and that the max-over-ranks timing reduction returns the slowest rank.
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import ROOT

sys.path.insert(0, str(ROOT))
import bench  # noqa: E402
from macboost_b200 import synth  # noqa: E402


class _Args:
    def __init__(self, scaling, rows=0):
        self.scaling = scaling
        self.rows = rows


@pytest.mark.parametrize("cfg", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_default_split_covers_the_workload(cfg, world):
    c = synth.CONFIGS[cfg]
    args = _Args(bench.default_scaling(c))
    rows = bench.rows_per_rank(c, args, world)
    assert rows % 4 == 0
    starts = [r * rows for r in range(world)]
    if cfg == "cfg5":
        assert args.scaling == "weak" and rows == c.rows // 8   # proportional slices
        assert starts[-1] + rows <= c.rows
    else:
        assert args.scaling == "strong"
        # contiguous, disjoint shards that cover the config's rows (the last may
        # reach past the end by less than 4 rows when rows % world != 0)
        assert rows * world >= c.rows and rows * (world - 1) < c.rows
        assert all(b - a == rows for a, b in zip(starts, starts[1:]))


def test_rank_slice_regenerates_the_same_rows():
    full = synth.make_data("cfg2", rows=50_000, layout="feature")
    for start, n in [(0, 12_500), (12_500, 12_500), (37_500, 12_500), (1_234, 4_321)]:
        part = synth.make_data("cfg2", rows=n, row_start=start, layout="feature")
        assert np.array_equal(part.view(np.uint32), full[:, start:start + n].view(np.uint32))


RANK_SCRIPT = textwrap.dedent(r"""
    import json, os, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1])
    import bench
    from macboost_b200 import synth
    from oracle import oracle as O
    import torch, torch.distributed as dist
    d = bench.Dist()
    cfg = synth.CONFIGS["cfg2"]
    class A: scaling = "strong"; rows = 0
    total = int(sys.argv[2])
    rows = (total // d.world + 3) // 4 * 4
    start = d.rank * rows
    rows = max(0, min(rows, total - start))
    X = synth.make_data(cfg, rows=rows, row_start=start, layout="feature")
    om = O.model_from_dict(json.loads(sys.argv[3]))
    raw = O.predict_raw(om, X, layout="feature", nthreads=1)
    parts = [None] * d.world
    dist.all_gather_object(parts, (start, raw.tolist()))
    slowest = d.max(float(d.rank + 1))
    d.barrier()
    if d.rank == 0:
        out = np.concatenate([np.asarray(p[1], np.float32) for p in sorted(parts)])
        np.save(sys.argv[4], out)
        print("MAX", slowest)
    d.close()
""")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_assemble_the_single_process_result(oracle_built, tmp_path):
    import json
    O = oracle_built
    total = 6_003
    text = synth.model_to_json(synth.make_model("cfg2", trees=24))
    out = tmp_path / "raw.npy"
    port = _free_port()
    procs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        procs.append(subprocess.Popen(
            [sys.executable, "-c", RANK_SCRIPT, str(ROOT), str(total), text, str(out)],
            env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, cwd=str(ROOT)))
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        assert p.returncode == 0, e[-2000:]
        outs.append(o)
    assert "MAX 2.0" in outs[0]
    whole = O.predict_raw(O.model_from_dict(json.loads(text)),
                          synth.make_data("cfg2", rows=total, layout="feature"), layout="feature")
    got = np.load(out)
    assert got.shape == whole.shape
    assert np.array_equal(got.view(np.uint32), whole.view(np.uint32))
