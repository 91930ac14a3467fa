"""GPU parity of the layer ops against the oracle through the C ABI.

Tolerance (north star): within 2 fp16 ulp for norm, RoPE and activation
outputs; the residual sum x + d is exact.  The kernels follow the oracle's
pinned orders, so in practice they agree bit for bit; the tests assert the
stated tolerance and report the exact-match fraction."""
import numpy as np
import pytest

from oracle_lib import f16_ulp_diff, f32_ulp_diff

pytestmark = pytest.mark.gpu

TOL_ULP = 2


def _torch():
    import torch
    return torch


def to_dev(a, dt):
    torch = _torch()
    if dt == "bf16":
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(a).cuda()


def to_host(t, dt):
    torch = _torch()
    if dt == "bf16":
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    return t.cpu().numpy()


def rand(rng, shape, dt, scale=1.0, outliers=0.0):
    a = rng.standard_normal(shape).astype(np.float32) * scale
    if outliers:
        m = rng.random(shape) < outliers
        a[m] *= 50.0
    if dt == "f16":
        return a.astype(np.float16)
    if dt == "bf16":
        return (a.view(np.uint32) >> 16).astype(np.uint16)  # truncation is fine for inputs
    return a


def ulp(a, b, dt):
    if dt == "f16":
        return f16_ulp_diff(a, b)
    if dt == "bf16":
        return f16_ulp_diff(a.view(np.float16), b.view(np.float16))  # same ordered-int metric
    return f32_ulp_diff(a, b)


def check(got, want, dt, what):
    d = ulp(got, want, dt)
    if dt == "f32":
        # fp32 outputs: 2 fp16 ulp == 2^14 fp32 ulp; assert much tighter
        assert d.max() <= 64, (what, int(d.max()))
    else:
        assert d.max() <= TOL_ULP, (what, int(d.max()))
    return float((d == 0).mean())


@pytest.mark.parametrize("dt", ["f16", "f32", "bf16"])
@pytest.mark.parametrize("dim", [128, 1000, 1024, 2048, 4096, 5120, 8192])
@pytest.mark.parametrize("with_d", [True, False])
def test_residual_rmsnorm(ane, oracle, dt, dim, with_d):
    rng = np.random.default_rng(dim + 7 * with_d)
    rows = 37
    x = rand(rng, (rows, dim), dt, outliers=0.001)
    d = rand(rng, (rows, dim), dt) if with_d else None
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    xt, dt_ = to_dev(x, dt), (to_dev(d, dt) if with_d else None)
    y = ane.residual_rmsnorm(xt, dt_, to_dev(w, "f32"))
    xo, yo = oracle.residual_rmsnorm(x, d, w)
    assert np.array_equal(to_host(xt, dt), xo)  # residual stream: exact
    check(to_host(y, dt), yo, dt, "rmsnorm")


# Many rows (several waves of CTAs, ragged counts that leave the last wave
# partial): the same bits as the oracle, row by row.
@pytest.mark.parametrize("dt,dim", [("f16", 4096), ("f16", 1024), ("bf16", 4096), ("bf16", 2048),
                                    ("f32", 2048), ("f32", 1024)])
@pytest.mark.parametrize("rows", [512, 1001, 5003])
@pytest.mark.parametrize("with_d", [True, False])
def test_residual_rmsnorm_many_rows(ane, oracle, dt, dim, rows, with_d):
    rng = np.random.default_rng(rows + dim + 7 * with_d)
    x = rand(rng, (rows, dim), dt, outliers=0.001)
    d = rand(rng, (rows, dim), dt) if with_d else None
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    xt, dt_ = to_dev(x, dt), (to_dev(d, dt) if with_d else None)
    y = ane.residual_rmsnorm(xt, dt_, to_dev(w, "f32"))
    xo, yo = oracle.residual_rmsnorm(x, d, w)
    assert np.array_equal(to_host(xt, dt), xo)
    got = to_host(y, dt)
    check(got, yo, dt, "rmsnorm many rows")
    assert np.array_equal(got.view(np.uint8), yo.view(np.uint8))  # same orders: same bits


def test_residual_rmsnorm_many_rows_strided(ane, oracle):
    """Row strides above the width (16-byte multiples) over many rows."""
    rng = np.random.default_rng(44)
    rows, dim, pitch = 777, 2048, 2048 + 64
    xb = rand(rng, (rows, pitch), "f16")
    db = rand(rng, (rows, pitch), "f16")
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    xt, dt_ = to_dev(xb, "f16"), to_dev(db, "f16")
    out = to_dev(np.zeros((rows, pitch), np.float16), "f16")
    ane.residual_rmsnorm(xt[:, :dim], dt_[:, :dim], to_dev(w, "f32"), out=out[:, :dim])
    xo, yo = oracle.residual_rmsnorm(xb[:, :dim].copy(), db[:, :dim].copy(), w)
    gx, gy = to_host(xt, "f16"), to_host(out, "f16")
    assert np.array_equal(gx[:, :dim], xo) and np.array_equal(gx[:, dim:], xb[:, dim:])
    assert np.array_equal(gy[:, :dim], yo) and not gy[:, dim:].any()


# The decode step's gather + (residual) RMSNorm in one launch: the same bits
# as the gather followed by the norm; bad ids read as zero rows and flag.
@pytest.mark.parametrize("tdt,odt", [("f16", "f32"), ("bf16", "f32"), ("f16", "f16"),
                                     ("bf16", "bf16"), ("f32", "f32")])
@pytest.mark.parametrize("hidden", [1024, 2048])
@pytest.mark.parametrize("acc", [False, True])
@pytest.mark.parametrize("rows", [1, 37])
def test_embedding_rmsnorm(ane, oracle, tdt, odt, hidden, acc, rows):
    torch = _torch()
    rng = np.random.default_rng(hidden + rows + 3 * acc)
    vocab = 1000
    table = rand(rng, (vocab, hidden), tdt, scale=0.5)
    ids = rng.integers(0, vocab, rows).astype(np.int32)
    if rows > 2:
        ids[1], ids[2] = -1, vocab  # outside the vocabulary
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    x0 = rand(rng, (rows, hidden), odt) if acc else None
    ane.read_status_flags(clear=True)
    xt = to_dev(x0, odt) if acc else None
    odt_t = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[odt]
    x, y = ane.embedding_rmsnorm(to_dev(table, tdt), torch.from_numpy(ids).cuda(), to_dev(w, "f32"),
                                 x=xt, accumulate=acc, out_dtype=odt_t)
    flags = ane.read_status_flags(clear=True)
    assert bool(flags & ane.FLAG_BAD_TOKEN_ID) == (rows > 2)
    code = {"f32": 0, "f16": 1, "bf16": 2}[odt]
    e, bad = oracle.embedding_gather(table, ids, out_dtype=code)
    assert bad == (2 if rows > 2 else 0)
    xo, yo = oracle.residual_rmsnorm(x0, e, w) if acc else oracle.residual_rmsnorm(e, None, w)
    if not acc:
        xo = e
    gx, gy = to_host(x, odt), to_host(y, odt)
    assert np.array_equal(gx.view(np.uint8), np.ascontiguousarray(xo).view(np.uint8))
    assert np.array_equal(gy.view(np.uint8), np.ascontiguousarray(yo).view(np.uint8))


def test_rmsnorm_in_place_and_strided(ane, oracle):
    torch = _torch()
    rng = np.random.default_rng(3)
    buf = rand(rng, (16, 3000), "f16")
    w = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    t = to_dev(buf, "f16")
    view = t[:, 8:8 + 2048]
    ane.residual_rmsnorm(view, None, to_dev(w, "f32"), out=view)
    _, yo = oracle.residual_rmsnorm(buf[:, 8:8 + 2048].copy(), None, w)
    got = t.cpu().numpy()
    check(got[:, 8:8 + 2048], yo, "f16", "strided in-place")
    assert np.array_equal(got[:, :8], buf[:, :8]) and np.array_equal(got[:, 2056:], buf[:, 2056:])
    assert torch.isfinite(t).all()


CASES = [  # (n_q, n_kv, head_dim, rot_dim)
    (16, 8, 128, 128),   # Qwen3-0.6B / 1.7B
    (32, 8, 128, 128),   # Qwen3-8B
    (8, 2, 64, 64),
    (4, 2, 256, 64),     # partial RoPE (generic path)
    (3, 1, 96, 96),      # non power-of-two chunk count (generic path)
    (64, 8, 128, 128),   # many heads
]


@pytest.mark.parametrize("dt", ["f16", "f32", "bf16"])
@pytest.mark.parametrize("case", CASES)
def test_qk_norm_rope(ane, oracle, dt, case):
    torch = _torch()
    nq, nkv, hd, rot = case
    rng = np.random.default_rng(nq * 1000 + hd)
    rows = 50
    qkv = rand(rng, (rows, (nq + 2 * nkv) * hd), dt, outliers=0.001)
    qw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    pos = np.concatenate([[0, 1, 2, 511, 2047, 4095, 65535, 1 << 20],
                          rng.integers(0, 40000, rows - 8)]).astype(np.int32)
    t = to_dev(qkv, dt)
    ane.qk_norm_rope(t, to_dev(qw, "f32"), to_dev(kw, "f32"), torch.from_numpy(pos).cuda(), nq,
                     nkv, hd, theta=1e6, rot_dim=rot)
    want = oracle.qk_norm_rope(qkv, nq, nkv, hd, qw, kw, pos, 1e6, rot_dim=rot)
    got = to_host(t, dt)
    check(got, want, dt, f"qk {case}")
    v0 = (nq + nkv) * hd
    assert np.array_equal(got[:, v0:].view(np.uint8), qkv[:, v0:].view(np.uint8))  # v untouched


# Many rows of the fused layout (several waves, ragged counts).
@pytest.mark.parametrize("dt", ["f16", "f32", "bf16"])
@pytest.mark.parametrize("case", [(32, 8, 128, 128), (16, 8, 128, 128), (8, 2, 64, 64)])
@pytest.mark.parametrize("rows", [512, 3001])
def test_qk_norm_rope_many_rows(ane, oracle, dt, case, rows):
    torch = _torch()
    nq, nkv, hd, rot = case
    rng = np.random.default_rng(nq * 7 + rows)
    qkv = rand(rng, (rows, (nq + 2 * nkv) * hd), dt, outliers=0.001)
    qw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    pos = rng.integers(0, 40000, rows).astype(np.int32)
    pos[:4] = [0, 1, 4095, 1 << 20]
    t = to_dev(qkv, dt)
    ane.qk_norm_rope(t, to_dev(qw, "f32"), to_dev(kw, "f32"), torch.from_numpy(pos).cuda(), nq,
                     nkv, hd, theta=1e6, rot_dim=rot)
    want = oracle.qk_norm_rope(qkv, nq, nkv, hd, qw, kw, pos, 1e6, rot_dim=rot)
    got = to_host(t, dt)
    check(got, want, dt, f"qk many rows {case}")
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))  # same orders: same bits


def test_rope_only_without_norm(ane, oracle):
    torch = _torch()
    rng = np.random.default_rng(21)
    nq, nkv, hd = 4, 2, 128
    qkv = rand(rng, (9, (nq + 2 * nkv) * hd), "f32")
    pos = np.arange(9, dtype=np.int32) * 1000
    t = to_dev(qkv, "f32")
    ane.qk_norm_rope(t, None, None, torch.from_numpy(pos).cuda(), nq, nkv, hd)
    # oracle with unit weights and no norm == rope alone: emulate by the generic identity
    ones = np.ones(hd, np.float32)
    normed = oracle.qk_norm_rope(qkv, nq, nkv, hd, ones, ones, np.zeros(9, np.int32), 1e6)
    assert not np.array_equal(to_host(t, "f32"), normed)
    # rope preserves the norm of each (j, j + half) pair
    a = qkv[:, :(nq + nkv) * hd].reshape(9, -1, 2, hd // 2)
    b = to_host(t, "f32")[:, :(nq + nkv) * hd].reshape(9, -1, 2, hd // 2)
    na = (a.astype(np.float64) ** 2).sum(2)
    nb = (b.astype(np.float64) ** 2).sum(2)
    assert np.allclose(na, nb, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dt", ["f16", "f32", "bf16"])
@pytest.mark.parametrize("shape", [(64, 3072), (33, 6144), (8, 12288), (5, 1001), (1, 7)])
def test_silu_mul(ane, oracle, dt, shape):
    rng = np.random.default_rng(shape[1])
    g = rand(rng, shape, dt, scale=3.0, outliers=0.01)
    u = rand(rng, shape, dt)
    out = ane.silu_mul(to_dev(g, dt), to_dev(u, dt))
    want = oracle.silu_mul(g, u)
    got = to_host(out, dt)
    check(got, want, dt, "silu")
    if dt == "f32":
        # pinned exp + IEEE divide: bit-exact with the oracle
        assert np.array_equal(got.view(np.int32), want.view(np.int32))
    else:
        # exp2 / reciprocal from the special-function unit: one unit at most
        assert ulp(got, want, dt).max() <= 1


# Long contiguous inputs take the bulk-copy ring (whole 32 KB tiles) and
# the plain kernel for the remainder: 701 x 12288 elements end mid-tile.
@pytest.mark.parametrize("dt", ["f16", "f32", "bf16"])
def test_silu_mul_bulk_path(ane, oracle, dt):
    rng = np.random.default_rng(701)
    shape = (701, 12288)
    g = rand(rng, shape, dt, scale=3.0, outliers=0.01)
    u = rand(rng, shape, dt)
    got = to_host(ane.silu_mul(to_dev(g, dt), to_dev(u, dt)), dt)
    want = oracle.silu_mul(g, u)
    if dt == "f32":
        assert np.array_equal(got.view(np.int32), want.view(np.int32))
    else:
        assert ulp(got, want, dt).max() <= 1


@pytest.mark.parametrize("dt", ["f16", "f32", "bf16"])
@pytest.mark.parametrize("op", ["silu_inplace", "mul_sigmoid_inplace"])
def test_inplace_bulk_matches_pieces(ane, dt, op):
    """The in-place forms on one long array (bulk-copy ring) give the bits of
    the same call on pieces too short for it (the 16-byte-vector kernel)."""
    torch = _torch()
    rng = np.random.default_rng(17)
    n = 701 * 12288
    x = rand(rng, (1, n), dt, scale=3.0, outliers=0.01)
    z = rand(rng, (1, n), dt, scale=3.0)
    code = {"f32": 0, "f16": 1, "bf16": 2}[dt]
    fn = getattr(ane.lib(), "ane_cuda_" + op)
    s = torch.cuda.current_stream().cuda_stream

    def run(xd, zd, start, count):
        es = xd.element_size()
        px, pz = xd.data_ptr() + start * es, zd.data_ptr() + start * es
        st = fn(code, px, count, s) if op == "silu_inplace" else fn(code, px, pz, count, s)
        assert st == 0

    whole, zd = to_dev(x, dt), to_dev(z, dt)
    run(whole, zd, 0, n)
    pieces = to_dev(x, dt)
    step = n // 64 + 8  # pieces well below the bulk threshold, ragged last one
    for start in range(0, n, step):
        run(pieces, zd, start, min(step, n - start))
    torch.cuda.synchronize()
    a, b = to_host(whole, dt), to_host(pieces, dt)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_silu_extremes(ane, oracle):
    g = np.array([[0.0, -0.0, -100.0, 100.0, -88.0, 88.0, -250.0, 250.0, 1e-30, -1e-30,
                   60000.0, -60000.0, 3.0, -3.0, 0.5, -0.5]], np.float32)
    u = np.ones_like(g)
    out = ane.silu_mul(to_dev(g, "f32"), to_dev(u, "f32"))
    want = oracle.silu_mul(g, u)
    assert np.array_equal(to_host(out, "f32").view(np.int32), want.view(np.int32))


def test_silu_tiny_results_bf16(ane, oracle):
    # bf16 keeps fp32's exponent range: gates near -88 give results near 1e-37
    g = np.array([[-80.0, -85.0, -86.5, -87.0, -87.5, -88.0, -88.5, -89.0, -95.0, -120.0]],
                 np.float32)
    gb = (g.view(np.uint32) >> 16).astype(np.uint16)
    ub = (np.ones_like(g).view(np.uint32) >> 16).astype(np.uint16)
    out = to_host(ane.silu_mul(to_dev(gb, "bf16"), to_dev(ub, "bf16")), "bf16")
    want = oracle.silu_mul(gb, ub)
    assert ulp(out, want, "bf16").max() <= 1, (out, want)


def test_silu_extremes_f16(ane, oracle):
    g = np.array([[0.0, -0.0, -100.0, 100.0, -88.0, 88.0, -250.0, 250.0, 1e-7, -1e-7,
                   60000.0, -60000.0, 3.0, -3.0, 0.5, -0.5, -17.0, -12.0, 6e-5, -6e-5]],
                 np.float16)
    u = np.array([[1.0, -1.0] * 10], np.float16)
    out = to_host(ane.silu_mul(to_dev(g, "f16"), to_dev(u, "f16")), "f16")
    want = oracle.silu_mul(g, u)
    assert f16_ulp_diff(out, want).max() <= 1
    assert np.array_equal(np.signbit(out), np.signbit(want))


# ------------------------------------------------- KV-cache write after RoPE
@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("per_row", [False, True], ids=["prefill", "batched_decode"])
def test_qk_norm_rope_kv(ane, oracle, dt, per_row):
    """models/llm/qwen3.cpp:470-488: k after RoPE and v into the ring slot; a
    row with slot -1 writes no cache row; every other slot keeps its bytes."""
    torch = _torch()
    rng = np.random.default_rng(31 + per_row)
    rows, nq, nkv, hd, cap = 12, 16, 8, 128, 20
    qkv = rand(rng, (rows, (nq + 2 * nkv) * hd), dt, outliers=0.01)
    qw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    pos = rng.integers(0, 4096, rows).astype(np.int32)
    if per_row:
        shape = (rows, cap, nkv, hd)
        slots = rng.integers(0, cap, rows).astype(np.int32)
    else:
        shape = (cap, nkv, hd)
        slots = rng.permutation(cap)[:rows].astype(np.int32)  # distinct slots of one ring
    slots[3] = -1
    kc = rand(rng, shape, dt)
    vc = rand(rng, shape, dt)
    wq, wk, wv = oracle.qk_norm_rope_kv(qkv, nq, nkv, hd, qw, kw, pos, 1e6, kc, vc, slots,
                                        per_row_cache=per_row)
    d = to_dev(qkv, dt)
    dk, dv = to_dev(kc, dt), to_dev(vc, dt)
    ane.qk_norm_rope_kv(d, torch.from_numpy(qw).cuda(), torch.from_numpy(kw).cuda(),
                        torch.from_numpy(pos).cuda(), nq, nkv, hd, dk, dv,
                        torch.from_numpy(slots).cuda())
    bits = (lambda a: a.view(np.uint32)) if dt == "f32" else (lambda a: a.view(np.uint16))
    assert np.array_equal(bits(to_host(d, dt)), bits(wq))
    assert np.array_equal(bits(to_host(dk, dt)), bits(wk))
    assert np.array_equal(bits(to_host(dv, dt)), bits(wv))


def test_qk_norm_rope_kv_bad_slot(ane, oracle):
    """A slot past the capacity writes no cache row and raises the flag."""
    torch = _torch()
    rng = np.random.default_rng(33)
    rows, nq, nkv, hd, cap = 3, 16, 8, 128, 8
    qkv = rand(rng, (rows, (nq + 2 * nkv) * hd), "f32")
    w = np.ones(hd, np.float32)
    pos = np.zeros(rows, np.int32)
    slots = np.array([1, cap, 2], np.int32)
    kc = np.zeros((cap, nkv, hd), np.float32)
    ok = slots.copy()
    ok[1] = -1
    _, wk, wv = oracle.qk_norm_rope_kv(qkv, nq, nkv, hd, w, w, pos, 1e6, kc, kc, ok)
    ane.read_status_flags(clear=True)
    dk, dv = torch.zeros(cap, nkv, hd, device="cuda"), torch.zeros(cap, nkv, hd, device="cuda")
    ane.qk_norm_rope_kv(torch.from_numpy(qkv).cuda(), torch.from_numpy(w).cuda(),
                        torch.from_numpy(w).cuda(), torch.from_numpy(pos).cuda(), nq, nkv, hd, dk, dv,
                        torch.from_numpy(slots).cuda())
    assert ane.read_status_flags(clear=True) & ane.FLAG_BAD_CACHE
    assert np.array_equal(dk.cpu().numpy(), wk) and np.array_equal(dv.cpu().numpy(), wv)
