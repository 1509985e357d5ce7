"""The N>1 bench path's host logic on CPU ranks (gloo, world size 2): rank 0 generates the cohort while rank 1 waits
for it; the ranks open it one after another; the job's time is its slowest rank's; the job's rate counts every rank's
windows (replicas, weak scaling); global_batch gathers every rank's windows and coordinates in rank order."""
import datetime
import os
import socket
import sys

import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, data, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), PANVRAM_B200_DATA=data)
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        import bench
        path, ds, _ = bench.ensure_cohort("cfg0", rank)
        ready = os.path.exists(os.path.join(path, "READY"))
        t = bench.max_over_ranks(0.5 + rank, world, "cpu")          # rank 1 is the slow one
        rate = bench.whole_job_rate(1024 * 10, world, t)
        import torch
        from panvram_b200.cohort import global_batch
        x = torch.full((3, 5), rank + 1, dtype=torch.uint8)
        co = torch.arange(12, dtype=torch.int64).view(3, 4) + 100 * rank
        X, Co = global_batch(x, co)
        gathered = (X[:, 0].tolist(), Co[:, 0].tolist())
        # the ranks' cohort opens, one at a time: each turn starts after the previous rank's has ended
        import time
        (t_start, t_end), _ = bench.one_rank_at_a_time(rank, world, lambda: (time.time(), (time.sleep(0.3), time.time())[1]))
        dist.barrier()
        q.put((rank, path, ds, ready, t, rate, gathered, (t_start, t_end)))
    finally:
        dist.destroy_process_group()


def test_two_cpu_ranks(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    (r0, path0, ds0, ready0, t0, rate0, g0, turn0), (r1, path1, ds1, ready1, t1, rate1, g1, turn1) = got
    assert turn1[0] >= turn0[1]                                     # rank 1's open began after rank 0's ended
    assert (r0, r1) == (0, 1)
    assert path0 == path1 == os.path.join(str(tmp_path), "cfg0") and ds0 == ds1 == "q4k"
    assert ready0 and ready1
    assert t0 == t1 == 1.5
    assert rate0 == rate1 == 2 * 1024 * 10 / 1.5
    # the global batch: every rank's rows, in rank order, on every rank
    assert g0 == g1 == ([1, 1, 1, 2, 2, 2], [0, 4, 8, 100, 104, 108])


def test_bench_parity_helpers():
    """bench.py's parity record: coordinates (assembly, contig index, start in the contig, strand) -> base-stream starts
    through the contig table, and mismatching rows counted against the CPU decoder's output."""
    import numpy as np
    import bench
    ctg = {"ctg_asm": np.array([0, 0, 1, 1, 1], np.int64), "ctg_boff": np.array([0, 100, 0, 50, 90], np.int64)}
    co = np.array([[0, 1, 7, 1], [1, 2, 3, 0], [1, 0, 0, 1]], np.int64)
    a, s, r = bench.coords_to_stream(ctg, co)
    assert a.tolist() == [0, 1, 1] and s.tolist() == [107, 93, 0] and r.tolist() == [1, 0, 1]

    def fn(asm, start, W, rc, tokens, verify=False):
        assert verify
        return np.stack([np.full(W, x % 256, np.uint8) for x in start])
    good = fn(a, s, 4, r, False, True)
    bad = good.copy()
    bad[1, 2] ^= 1
    par = bench.parity_check(fn, "reference", [(good, a, s, r), (bad, a, s, r)], 4, False)
    assert par["windows"] == 6 and par["mismatches"] == 1 and par["first_mismatch"] == {"asm": 1, "start": 93}
