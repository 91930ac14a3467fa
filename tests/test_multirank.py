"""Multi-rank host logic of bench.py on the CPU, as gloo ranks (world size 2).

The layer-op path shards by rows with no collective on the data path: each
rank owns a disjoint block of global rows and generates its inputs from the
seed and its row offset.  Checked here: the blocks tile the global rows;
results computed rank by rank (by the oracle, standing in for the kernels on
a machine without a GPU) equal one single-process run over all the rows;
the timing collective returns the slowest rank's time on every rank; the
whole-job figure counts every rank's rows; the reference arm runs on rank 0
only.  The gather below is test scaffolding, not part of the path."""
import contextlib
import datetime
import io
import multiprocessing as mp
import os
import socket
import time

import numpy as np

WORLD = 2
ROWS_PER_RANK = 6
HIDDEN, NQ, NKV, HD, INTER = 256, 4, 2, 64, 384


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def block_inputs(bench, row0, n):
    """A rank's inputs: fp16 rows seeded by bench.chain_seed(row0)."""
    rng = np.random.default_rng(bench.chain_seed(row0))
    f16 = lambda *s: rng.standard_normal(s).astype(np.float16)  # noqa: E731
    return {"x": f16(n, HIDDEN), "d": f16(n, HIDDEN), "qkv": f16(n, (NQ + 2 * NKV) * HD),
            "gate": f16(n, INTER), "up": f16(n, INTER),
            "pos": ((row0 + np.arange(n)) % 512).astype(np.int32)}


def chain(oracle, b, w, qw, kw):
    x, y = oracle.residual_rmsnorm(b["x"], b["d"], w)
    q = oracle.qk_norm_rope(b["qkv"], NQ, NKV, HD, qw, kw, b["pos"], 1e6)
    h = oracle.silu_mul(b["gate"], b["up"])
    return np.concatenate([x, y, q, h], axis=1)


def weights():
    rng = np.random.default_rng(7)
    return ((1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32),
            (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32),
            (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32))


def _rank_main(rank, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      LOCAL_RANK=str(rank), WORLD_SIZE=str(WORLD))
    import torch.distributed as dist
    import torch

    import bench
    from oracle_lib import Oracle
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    try:
        r, lr, wsz = bench.env_rank()
        row0, n = bench.rank_rows(r, ROWS_PER_RANK)
        res = chain(Oracle(), block_inputs(bench, row0, n), *weights())
        slowest = bench.max_over_ranks(torch, dist, wsz, 1.5 + rank)
        # the reference arm: rank 0 alone runs it; other ranks return at once
        quiet = None
        if r != 0:
            buf = io.StringIO()
            t0 = time.perf_counter()
            with contextlib.redirect_stdout(buf):
                bench.run_reference(None)
            quiet = (buf.getvalue() == "", time.perf_counter() - t0)
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, (r, lr, wsz, row0, n, res, slowest, quiet))
        if r == 0:
            out_q.put(gathered)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_rows_without_a_data_path_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
    for p in procs:
        assert p.exitcode == 0
    got.sort(key=lambda t: t[0])
    import bench
    from oracle_lib import Oracle
    # rank identity from the launcher's environment
    assert [(g[0], g[1], g[2]) for g in got] == [(r, r, WORLD) for r in range(WORLD)]
    # disjoint blocks that tile rows [0, WORLD * R)
    spans = [(g[3], g[4]) for g in got]
    assert spans == [(r * ROWS_PER_RANK, ROWS_PER_RANK) for r in range(WORLD)]
    # per-rank results == one run over all rows (rows are independent)
    allb = [block_inputs(bench, r0, n) for r0, n in spans]
    merged = {k: np.concatenate([b[k] for b in allb]) for k in allb[0]}
    want = chain(Oracle(), merged, *weights())
    have = np.concatenate([g[5] for g in got])
    assert np.array_equal(have.view(np.uint16), want.view(np.uint16))
    # the timing collective: the slowest rank's value on every rank
    assert all(g[6] == 1.5 + (WORLD - 1) for g in got)
    # whole-job throughput counts every rank's rows over the slowest time
    one = bench.aggregate_gbs(1, bench.ROWS, 1.0)
    assert abs(bench.aggregate_gbs(WORLD, bench.ROWS, 1.0) - WORLD * one) < 1e-9
    # the reference arm printed nothing on rank 1 and returned at once
    quiet, dt = got[1][7]
    assert quiet and dt < 1.0
