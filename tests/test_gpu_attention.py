"""GPU decode attention over a ring KV cache (core/cpu_ops.cpp:173-240)
through the C ABI.

fp32 caches: the CUDA-core kernel takes every sum in the oracle's fixed
order, so the two agree bit for bit.  16-bit caches: the contractions run on
the tensor cores, whose internal summation order is the hardware's, and the
softmax is taken online over each warp's keys; the fp32 result is then
within about 1e-6 relative of the oracle's, so the stored
fp16 / bf16 outputs agree with the oracle's to within one unit in the last
place (most of them exactly).  Against the reference itself (its
gqa_attention compiled with the shim, sequential sums) the fp32 output must
be within 1e-6 x max|v| -- the two summation orders each stay within about
1e-7 x max|v| of the exact (fp64) result."""
import zlib

import numpy as np
import pytest

from test_gpu_layer_ops import rand, to_dev, to_host

pytestmark = pytest.mark.gpu

REF_TOL = 1e-6  # x max|v|, fp32 vs the reference's sequential sums


def _torch():
    import torch
    return torch


def make_case(rng, B, H, hk, hd, cap, starts, lens, dt):
    q = rand(rng, (B, H, hd), dt)
    k = rand(rng, (B, cap, hk, hd), dt)
    v = rand(rng, (B, cap, hk, hd), dt)
    return q, k, v, np.array(starts, np.int32), np.array(lens, np.int32)


def run_gpu(ane, q, k, v, st, ln, dt, max_len=None, workspace=None):
    torch = _torch()
    out = ane.decode_attention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt),
                               torch.from_numpy(st).cuda(), torch.from_numpy(ln).cuda(),
                               max_len=max_len, workspace=workspace)
    torch.cuda.synchronize()
    return to_host(out, dt)


def bits(a):
    return a.view(np.uint32) if a.dtype == np.float32 else a.view(np.uint16)


# 16-bit outputs (tensor-core contractions): one unit of the output type,
# plus an absolute 1e-5 x max|v| for outputs near zero, where the fp32
# difference (P kept to 2^-17 relative in bf16, 2^-22 in fp16) spans several
# units of a small value.
ABS_TOL = 1e-5


def as_f32(a, dt):
    if dt == "bf16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def unit(want32, dt):
    """One unit in the last place of each fp16 / bf16 value (normal range)."""
    if dt == "f16":
        return np.spacing(np.abs(want32).astype(np.float16)).astype(np.float32)
    e = (want32.view(np.uint32) >> 23) & 0xFF
    return np.ldexp(np.float32(1), np.maximum(e.astype(np.int32) - 127 - 7, -133)).astype(np.float32)


def check_against_oracle(got, want, dt, vmax=1.0):
    if dt == "f32":
        assert np.array_equal(bits(got), bits(want)), (
            f"{int((bits(got) != bits(want)).sum())} of {got.size} differ")
        return
    g32, w32 = as_f32(got, dt), as_f32(want, dt)
    err = np.abs(g32 - w32)
    lim = unit(w32, dt) + np.float32(ABS_TOL * vmax)
    assert np.all(err <= lim), (float((err / lim).max()), int((err > lim).sum()), got.size)
    assert (bits(got) == bits(want)).mean() > 0.9


SHAPES = [
    # B, H, Hk, hd, cap, starts, lens
    (1, 16, 8, 128, 4096, [0], [4096]),      # Qwen3-0.6B, full ring
    (1, 16, 8, 128, 4096, [1000], [4096]),   # full ring, wrapped
    (1, 16, 8, 128, 4096, [4000], [200]),    # wraps inside the window
    (1, 16, 8, 128, 512, [3], [1]),          # one key
    (1, 16, 8, 128, 512, [0], [64]),         # exactly one split
    (1, 16, 8, 128, 512, [0], [65]),         # one key into the second split
    (1, 32, 8, 128, 300, [250], [290]),      # Qwen3-8B grouping, odd capacity
    (1, 40, 8, 128, 256, [17], [255]),       # 5 q heads per kv head
    (1, 8, 8, 64, 100, [99], [37]),          # head_dim 64, no grouping
    (1, 24, 8, 64, 1000, [5], [999]),        # 3 q heads per kv head
    (1, 16, 2, 256, 129, [5], [129]),        # head_dim 256, 8 per kv head
    (3, 16, 8, 128, 700, [0, 650, 13], [700, 0, 333]),  # batch, an empty sequence
]


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"B{s[0]}H{s[1]}k{s[2]}d{s[3]}c{s[4]}")
def test_attention_matches_oracle(ane, oracle, dt, shape):
    B, H, hk, hd, cap, starts, lens = shape
    rng = np.random.default_rng(zlib.crc32(repr((B, H, hk, hd, cap, dt)).encode()))
    q, k, v, st, ln = make_case(rng, B, H, hk, hd, cap, starts, lens, dt)
    want = oracle.decode_attention(q, k, v, st, ln)
    got = run_gpu(ane, q, k, v, st, ln, dt)
    check_against_oracle(got, want, dt, float(np.abs(as_f32(v, dt) if dt != "f32" else v).max()))


# Batches large enough that the 16-bit kernel takes several 64-key chunks
# per CTA: one split per (kv head, sequence) with the copy ring reused many
# times (first three), or a few splits of several chunks each (last two);
# lengths ragged from 0 to the capacity, starts anywhere in the ring.
PIPE_SHAPES = [
    # B, H, Hk, hd, cap
    (40, 32, 8, 128, 777),
    (40, 16, 8, 64, 600),
    (24, 64, 8, 256, 333),
    (12, 32, 8, 128, 1000),
    (8, 32, 8, 128, 2048),
]


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("shape", PIPE_SHAPES, ids=lambda s: f"B{s[0]}H{s[1]}k{s[2]}d{s[3]}c{s[4]}")
def test_attention_long_splits(ane, oracle, dt, shape):
    B, H, hk, hd, cap = shape
    rng = np.random.default_rng(zlib.crc32(repr(("pipe", shape, dt)).encode()))
    lens = rng.integers(1, cap + 1, size=B)
    special = [0, 1, 64, 65, cap, cap - 1]
    lens[:len(special)] = special
    starts = rng.integers(0, cap, size=B)
    q, k, v, st, ln = make_case(rng, B, H, hk, hd, cap, starts, lens, dt)
    want = oracle.decode_attention(q, k, v, st, ln)
    got = run_gpu(ane, q, k, v, st, ln, dt)
    check_against_oracle(got, want, dt, float(np.abs(as_f32(v, dt) if dt != "f32" else v).max()))


@pytest.mark.parametrize("shape", SHAPES[:9], ids=lambda s: f"H{s[1]}k{s[2]}d{s[3]}c{s[4]}l{s[6][0]}")
def test_attention_matches_reference(ane, ref, shape):
    B, H, hk, hd, cap, starts, lens = shape
    rng = np.random.default_rng(7)
    q, k, v, st, ln = make_case(rng, B, H, hk, hd, cap, starts, lens, "f32")
    got = run_gpu(ane, q, k, v, st, ln, "f32")
    want = np.empty_like(q[0])
    from oracle_lib import _ptr
    ref.ref_gqa_attention(_ptr(want), _ptr(q[0]), _ptr(np.ascontiguousarray(k[0])),
                          _ptr(np.ascontiguousarray(v[0])), H, hk, hd, hd, int(st[0]), int(ln[0]),
                          cap)
    tol = REF_TOL * np.abs(v).max()
    assert np.abs(got[0] - want).max() <= tol


# fp32, one sequence alone and the same sequence as row 17 of a batch of
# 40 with other lengths and starts: both give the oracle's bits (a split's
# partials and the merge do not depend on the other rows of the batch).
# Lengths ragged against the 64-key splits, wrapped rings, 8192 keys, 8 q
# heads per kv head, head_dim 64, max_len below the capacity.
BATCH_POSITION_CASES = [
    # H, Hk, hd, cap, start, len, max_len
    (16, 8, 128, 4096, 0, 4096, None),
    (16, 8, 128, 4096, 1000, 4000, None),
    (16, 8, 128, 8192, 77, 8192, None),
    (16, 8, 128, 1024, 1000, 129, None),
    (16, 8, 128, 4096, 5, 700, 1000),
    (64, 8, 128, 2048, 2000, 2047, None),
    (32, 8, 64, 3000, 2999, 3000, None),
    (24, 8, 128, 512, 500, 300, None),
]


@pytest.mark.parametrize("case", BATCH_POSITION_CASES, ids=lambda c: f"H{c[0]}k{c[1]}d{c[2]}c{c[3]}l{c[5]}")
def test_attention_same_bits_alone_and_in_a_batch(ane, oracle, case):
    H, hk, hd, cap, start, length, max_len = case
    rng = np.random.default_rng(zlib.crc32(repr(("cl", case)).encode()))
    q, k, v, st, ln = make_case(rng, 1, H, hk, hd, cap, [start], [length], "f32")
    want = oracle.decode_attention(q, k, v, st, ln)
    one = run_gpu(ane, q, k, v, st, ln, "f32", max_len=max_len)
    assert np.array_equal(bits(one), bits(want)), int((bits(one) != bits(want)).sum())
    B = 40  # the sequence as row 17 of a batch
    qb, kb_, vb, stb, lnb = make_case(rng, B, H, hk, hd, cap, list(rng.integers(0, cap, B)),
                                      list(rng.integers(1, length + 1, B)), "f32")
    qb[17], kb_[17], vb[17], stb[17], lnb[17] = q[0], k[0], v[0], st[0], ln[0]
    many = run_gpu(ane, qb, kb_, vb, stb, lnb, "f32", max_len=max_len)
    assert np.array_equal(bits(many[17]), bits(one[0]))


def test_attention_caller_workspace_two_calls(ane, oracle):
    """A caller workspace full of garbage (it needs no clearing: only the
    call in flight keeps its split partials there) gives the same bits as
    the library-held one, twice in a row."""
    torch = _torch()
    rng = np.random.default_rng(11)
    B, H, hk, hd, cap = 2, 16, 8, 128, 1024
    q, k, v, st, ln = make_case(rng, B, H, hk, hd, cap, [100, 0], [1024, 517], "f32")
    want = oracle.decode_attention(q, k, v, st, ln)
    nbytes = ane.decode_attention_workspace_size(B, H, hk, hd, cap)
    assert nbytes > 0
    ws = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        got = run_gpu(ane, q, k, v, st, ln, "f32", workspace=ws)
        assert np.array_equal(bits(got), bits(want))
    got = run_gpu(ane, q, k, v, st, ln, "f32")
    assert np.array_equal(bits(got), bits(want))


def test_attention_workspace_reused_across_shapes(ane, oracle):
    """One workspace (the caller's, then the library's own) serving calls of
    different shapes in turn: each call's partials land where the previous
    call of another shape kept its own.  Every call must still give the
    oracle's bits."""
    torch = _torch()
    rng = np.random.default_rng(77)
    cases = [(1, 16, 8, 128, 4096, [9], [4096]),
             (16, 32, 8, 128, 1024, list(rng.integers(0, 1024, 16)), list(rng.integers(1, 1025, 16))),
             (2, 16, 8, 128, 2048, [100, 7], [2048, 1500]),
             (16, 32, 8, 128, 1024, list(rng.integers(0, 1024, 16)), list(rng.integers(1, 1025, 16)))]
    size = max(ane.decode_attention_workspace_size(B, H, hk, hd, cap) for B, H, hk, hd, cap, _, _ in cases)
    ws = torch.zeros(size, dtype=torch.uint8, device="cuda")
    for workspace in (ws, None):
        for B, H, hk, hd, cap, starts, lens in cases:
            q, k, v, st, ln = make_case(rng, B, H, hk, hd, cap, starts, lens, "f32")
            want = oracle.decode_attention(q, k, v, st, ln)
            got = run_gpu(ane, q, k, v, st, ln, "f32", workspace=workspace)
            assert np.array_equal(bits(got), bits(want)), (B, H, cap, workspace is None)


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_attention_graph_replay_between_other_shapes(ane, oracle, dt):
    """A call captured in a CUDA graph, replayed after eager calls of other
    shapes on the same workspace (whose partials cover the captured call's
    part of it) and after a replay of another graph: every replay gives the
    same bits as the eager call."""
    torch = _torch()
    rng = np.random.default_rng(31)
    X = (1, 16, 8, 128, 4096, [1000], [4096])
    Y = (16, 32, 8, 128, 1024, list(rng.integers(0, 1024, 16)), list(rng.integers(1, 1025, 16)))
    size = max(ane.decode_attention_workspace_size(B, H, hk, hd, cap) for B, H, hk, hd, cap, _, _ in (X, Y))
    ws = torch.full((size,), 0x7F, dtype=torch.uint8, device="cuda")

    def dev_case(c):
        B, H, hk, hd, cap, starts, lens = c
        host = make_case(rng, B, H, hk, hd, cap, starts, lens, dt)
        d = [to_dev(a, dt) for a in host[:3]] + [torch.from_numpy(a).cuda() for a in host[3:]]
        return host, d, torch.empty_like(d[0])

    (hx, dx, ox), (hy, dy, oy) = dev_case(X), dev_case(Y)
    want_x = oracle.decode_attention(*hx)
    vmax = float(np.abs(as_f32(hx[2], dt)).max())
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ane.decode_attention(*dx, out=ox, workspace=ws)  # eager warm-up of X
        s.synchronize()
        eager_x = to_host(ox.clone(), dt)
        gx, gy = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(gx, stream=s):
            ane.decode_attention(*dx, out=ox, workspace=ws)
        with torch.cuda.graph(gy, stream=s):
            ane.decode_attention(*dy, out=oy, workspace=ws)
        for order in ("eager_y", "replay_y", "both"):
            ox.zero_()
            if order in ("eager_y", "both"):
                ane.decode_attention(*dy, out=oy, workspace=ws)
            if order in ("replay_y", "both"):
                gy.replay()
            gx.replay()
            s.synchronize()
            got = to_host(ox, dt)
            assert np.array_equal(bits(got), bits(eager_x)), order
        del gx, gy
    check_against_oracle(eager_x, want_x, dt, vmax)


def test_attention_held_workspace_not_grown_during_capture(ane, oracle):
    """The library-held workspace of a stream is never allocated during a
    stream capture: such a call is refused with a clear error (the capture
    itself stays valid), and after one eager call of the shape the same
    capture works and replays to the oracle's bits."""
    torch = _torch()
    rng = np.random.default_rng(41)
    host = make_case(rng, 1, 16, 8, 128, 4096, [5], [4096], "f32")
    want = oracle.decode_attention(*host)
    d = [to_dev(a, "f32") for a in host[:3]] + [torch.from_numpy(a).cuda() for a in host[3:]]
    out = torch.empty_like(d[0])
    # max_len far above the keys sizes a workspace (about 136 MB) larger
    # than any earlier call gave a pooled stream, so this call must grow it
    big = 1 << 20
    assert ane.decode_attention_workspace_size(1, 16, 8, 128, big) > 100 << 20
    s = torch.cuda.Stream()
    err = None
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            try:
                ane.decode_attention(*d, out=out, max_len=big)
            except ane.AneCudaError as e:
                err = e
        assert err is not None and err.status == ane.ERR_INVALID_ARG
        assert "capture" in str(err)
        del g
        ane.decode_attention(*d, out=out, max_len=big)  # eager: grows the stream's workspace
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ane.decode_attention(*d, out=out, max_len=big)
        out.zero_()
        g.replay()
        s.synchronize()
        assert np.array_equal(bits(to_host(out, "f32")), bits(want))
        del g


def test_attention_max_len_sizes_launch(ane, oracle):
    """max_len below the capacity launches fewer splits; same bits."""
    rng = np.random.default_rng(12)
    q, k, v, st, ln = make_case(rng, 1, 16, 8, 128, 4096, [4090], [300], "f16")
    want = oracle.decode_attention(q, k, v, st, ln)
    got = run_gpu(ane, q, k, v, st, ln, "f16", max_len=300)
    check_against_oracle(got, want, "f16", float(np.abs(v.astype(np.float32)).max()))
    again = run_gpu(ane, q, k, v, st, ln, "f16", max_len=300)
    assert np.array_equal(bits(got), bits(again))  # deterministic


def test_attention_bad_cache_flag(ane):
    """len > max_len or > capacity, or start outside: zeros and a flag."""
    rng = np.random.default_rng(13)
    ane.read_status_flags(clear=True)
    q, k, v, st, ln = make_case(rng, 3, 16, 8, 128, 256, [0, 300, 0], [100, 10, 257], "f32")
    got = run_gpu(ane, q, k, v, st, ln, "f32", max_len=256)
    flags = ane.read_status_flags(clear=True)
    assert flags & ane.FLAG_BAD_CACHE
    assert not np.any(got[1]) and not np.any(got[2])
    assert np.any(got[0])


def test_attention_rejects_unsupported(ane):
    torch = _torch()
    q = torch.zeros((1, 16, 96), device="cuda")
    k = torch.zeros((1, 64, 8, 96), device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ane.AneCudaError) as e:
        ane.decode_attention(q, k, k, st, st)
    assert e.value.status == ane.ERR_UNSUPPORTED
    q = torch.zeros((1, 32, 128), device="cuda")
    k = torch.zeros((1, 64, 2, 128), device="cuda")  # 16 q heads per kv head
    with pytest.raises(ane.AneCudaError):
        ane.decode_attention(q, k, k, st, st)
