"""Multi-rank host logic of bench.py on the CPU, as gloo ranks (world size 2).

The layer-op path shards by rows with no collective on the data path: the
fixed global batch is split into contiguous blocks (sizes differing by at
most one), and each rank generates its block's inputs from per-sequence
seeds, so the global inputs do not depend on the number of ranks.  Checked
here, with an uneven split (13 rows over 2 ranks, sequences of 4 rows that
straddle the rank boundary): the blocks tile the global rows; each rank's
inputs equal the matching rows of a single-process batch; results computed
rank by rank (by the oracle, standing in for the kernels on a machine
without a GPU) equal one single-process run over all the rows; the timing
collective returns the slowest rank's values on every rank; the whole-job
figure counts the global rows once; the reference arm runs on rank 0 only.
The gather below is test scaffolding, not part of the path."""
import contextlib
import datetime
import io
import multiprocessing as mp
import os
import socket
import time

import numpy as np

WORLD = 2
TOTAL = 13
SEQ = 4
HIDDEN, NQ, NKV, HD, INTER = 256, 4, 2, 64, 384


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def block_inputs(bench, row0, n):
    """Rows [row0, row0 + n) of the global batch, as bench.py builds them
    (torch on the CPU here), converted to numpy."""
    import torch
    b = bench.make_chain_inputs(torch, row0, n, HIDDEN, NQ, NKV, HD, INTER, SEQ, device="cpu")
    return {k: v.numpy() for k, v in b.items()}


def chain(oracle, b):
    x, y = oracle.residual_rmsnorm(b["x"], b["d"], b["w"])
    q = oracle.qk_norm_rope(b["qkv"], NQ, NKV, HD, b["qw"], b["kw"], b["pos"], 1e6)
    h = oracle.silu_mul(b["gate"], b["up"])
    return np.concatenate([x, y, q, h], axis=1)


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
        row0, n = bench.rank_rows(r, wsz, TOTAL)
        b = block_inputs(bench, row0, n)
        res = chain(Oracle(), b)
        slowest = bench.max_over_ranks(torch, dist, wsz, [1.5 + rank, 7.0 - rank])
        one = bench.max_over_ranks(torch, dist, wsz, 2.0 * (rank + 1))
        # the reference arm: rank 0 alone runs it; other ranks return at once
        quiet = None
        if r != 0:
            buf = io.StringIO()
            t0 = time.perf_counter()
            with contextlib.redirect_stdout(buf):
                bench.run_reference(None)
            quiet = (buf.getvalue() == "", time.perf_counter() - t0)
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, (r, lr, wsz, row0, n, b, res, slowest, one, quiet))
        if r == 0:
            out_q.put(gathered)
    finally:
        dist.destroy_process_group()


def test_row_blocks_are_contiguous_and_balanced():
    import bench
    for total in (1, 7, 13, 256, 32768, bench.CONVERT_PARAMS):
        for world in (1, 2, 3, 4, 8):
            spans = [bench.rank_rows(r, world, total) for r in range(world)]
            assert spans[0][0] == 0
            assert all(a[0] + a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert spans[-1][0] + spans[-1][1] == total
            sizes = [n for _, n in spans]
            assert max(sizes) - min(sizes) <= 1
    # BASELINE config 3 at 8 GPUs: 4096 rows (8 whole sequences) per rank
    assert bench.rank_rows(7, 8) == (7 * 4096, 4096)


def test_rotation_sets_cover_more_than_l2():
    import bench
    for world in (1, 2, 4, 8):
        _, n = bench.rank_rows(0, world)
        sb = bench.chain_set_bytes(n, bench.HIDDEN, bench.NQ, bench.NKV, bench.HD, bench.INTER)
        k = bench.rotation_sets(sb)
        assert k * sb >= bench.ROTATE_BYTES
        # between two launches of one kernel on one set, the other sets and
        # kernels stream more than 4 L2s
        reuse = k * n * bench.B_ROW - n * max(bench.B_NORM, bench.B_QK, bench.B_SILU)
        assert reuse > 4 * 126e6


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
    # uneven contiguous blocks that tile rows [0, TOTAL)
    spans = [(g[3], g[4]) for g in got]
    assert spans == [(0, 6), (6, 7)]
    # each rank's inputs are the matching rows of the single-process batch
    whole = block_inputs(bench, 0, TOTAL)
    for (r0, n), g in zip(spans, got):
        for k in ("x", "d", "qkv", "gate", "up", "pos"):
            assert np.array_equal(g[5][k], whole[k][r0:r0 + n]), k
        for k in ("w", "qw", "kw"):
            assert np.array_equal(g[5][k], whole[k]), k
    # per-rank results == one run over all rows (rows are independent)
    want = chain(Oracle(), whole)
    have = np.concatenate([g[6] for g in got])
    assert np.array_equal(have.view(np.uint16), want.view(np.uint16))
    # the timing collective: the slowest rank's values on every rank
    assert all(g[7] == [2.5, 7.0] for g in got)
    assert all(g[8] == 4.0 for g in got)
    # whole-job throughput counts the global rows once, over the slowest time
    assert abs(bench.aggregate_gbs(bench.ROWS, 1.0) - bench.ROWS * bench.B_ROW / 1e6) < 1e-6
    # the reference arm printed nothing on rank 1 and returned at once
    quiet, dt = got[1][9]
    assert quiet and dt < 1.0


def test_per_kernel_events_on_a_subset_of_steps():
    import bench
    for steps in (1, 2, 3, 4, 20, 200):
        marked = [i for i in range(steps) if bench.instrumented(i, steps)]
        assert marked and len(marked) <= max(1, steps // bench.EVENT_EVERY)
        assert all(0 <= i < steps for i in marked)
