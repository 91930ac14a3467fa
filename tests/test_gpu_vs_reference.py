"""The GPU kernels checked directly against the REFERENCE's own CPU code
(oracle/_ref: core/cpu_ops.cpp, core/sampling.cpp compiled with the shim),
at BASELINE's shapes, and against the fixtures that build wrote
(tests/golden/rmsnorm.npz, qk_rope.npz, silu.npz).

- fp16 layer chain (configs 2 and 3: residual + RMSNorm, QK-norm + RoPE,
  SiLU-gate; models/llm/qwen3.cpp:444-473, :516-518; core/cpu_ops.cpp:7-31,
  :43-54) against ref_layer_chain_f16 over 256 rows with 0.1% x50 outliers:
  the residual bit-exact, every other output within 2 fp16 ulp (the
  north star's bound), the exact-match fraction printed.
- config 1's fp32 decode chain (gather from the fp16 table, fp32 residual
  RMSNorm, per-head QK-norm + RoPE at a position below 4096 on the model's
  libm cos/sin table, SiLU(gate) * up): gather bit-exact; the rest within
  2 fp16 ulp of the reference, and in fp32 ulps as printed.
- sample_token with non-finite logits (+Inf, NaN, -inf masks, all -inf,
  overflow under 1/T), all-equal rows and greedy ties: token ids equal.
- softmax on the same rows: NaN where the reference has NaN, every other
  value bit-exact.
- apply_rope_cached without tables (the reference's interleaved fallback,
  core/cpu_ops.cpp:66-77): bit-exact against the restatement, within
  1e-6 x max|v| of the reference."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle_lib import f16_ulp_diff, f32_ulp_diff

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def _t():
    import torch
    return torch


def dev(a):
    return _t().from_numpy(np.ascontiguousarray(a)).cuda()


def f16_act(rng, shape):
    a = rng.standard_normal(shape).astype(np.float32)
    a[rng.random(shape) < 1e-3] *= 50.0
    return a.astype(np.float16)


def within_2_f16_ulp(got32, want32):
    """|got - want| <= 2 ulp of fp16 at |want| (fp32 outputs)."""
    ulp = np.spacing(np.abs(want32).astype(np.float16)).astype(np.float32)
    return np.abs(got32.astype(np.float32) - want32.astype(np.float32)) <= 2 * ulp


# --------------------------------------------------------------- fp16 chain
@pytest.mark.parametrize("shape", [
    ("qwen3-8b", 4096, 32, 8, 128, 12288, 512),    # config 3: positions row mod 512
    ("qwen3-1.7b", 2048, 16, 8, 128, 6144, 2048),  # config 2: positions 0..2047
], ids=lambda s: s[0])
def test_fp16_chain_vs_reference(ane, ref, shape):
    name, hidden, nq, nkv, hd, inter, seq = shape
    rows = 256
    rng = np.random.default_rng(hidden)
    x = f16_act(rng, (rows, hidden))
    d = f16_act(rng, (rows, hidden))
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    qkv = f16_act(rng, (rows, (nq + 2 * nkv) * hd))
    qw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    # rows spread over the sequence: positions 0..seq-1 all reachable
    pos = (np.arange(rows) * (seq // rows if seq > rows else 1) + rng.integers(0, 2, rows)) % seq
    pos = pos.astype(np.int32)
    pos[:4] = [0, 1, seq - 1, seq // 2]
    g = f16_act(rng, (rows, inter))
    u = f16_act(rng, (rows, inter))

    xr, yr, qr, hr = x.copy(), np.empty_like(x), qkv.copy(), np.empty_like(g)
    ref.ref_layer_chain_f16(ptr(xr), ptr(d), ptr(yr), ptr(w), ptr(qr), ptr(qw), ptr(kw), ptr(pos),
                            ptr(g), ptr(u), ptr(hr), 0, rows, hidden, nq, nkv, hd, inter,
                            np.float32(1e6), np.float32(1e-6))

    xt, qt = dev(x), dev(qkv)
    yt = ane.residual_rmsnorm(xt, dev(d), dev(w))
    ane.qk_norm_rope(qt, dev(qw), dev(kw), dev(pos), nq, nkv, hd, theta=1e6)
    ht = ane.silu_mul(dev(g), dev(u))
    _t().cuda.synchronize()
    xg, yg, qg, hg = (t.cpu().numpy() for t in (xt, yt, qt, ht))

    assert np.array_equal(xg.view(np.uint16), xr.view(np.uint16)), "residual"
    qk = slice(0, (nq + nkv) * hd)
    for nm, got, want in (("rmsnorm", yg, yr), ("qk_norm_rope", qg[:, qk], qr[:, qk]),
                          ("silu_mul", hg, hr)):
        ulps = f16_ulp_diff(got, want)
        exact = float((ulps == 0).mean())
        print(f"{name} {nm}: max {int(ulps.max())} fp16 ulp, {100 * exact:.3f}% bit-exact")
        assert ulps.max() <= 2, (nm, int(ulps.max()))
    # the v heads are not touched
    assert np.array_equal(qg[:, (nq + nkv) * hd:].view(np.uint16), qkv[:, (nq + nkv) * hd:].view(np.uint16))


# --------------------------------------------------------------- fp32 decode chain
def test_fp32_decode_chain_vs_reference(ane, ref):
    """BASELINE config 1 (Qwen3-0.6B, batch 1): token id ~U[0,151936), fp16
    table N(0, 0.02), fp32 residual N(0, 1), norm weights 1 + N(0, 0.1),
    16 / 8 heads of 128, position ~U[0, 4096), gate / up N(0, 1) over 3072."""
    torch = _t()
    rng = np.random.default_rng(2025)
    vocab, hidden, nq, nkv, hd, inter = 151936, 1024, 16, 8, 128, 3072
    for trial in range(4):
        table = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float16)
        tok = np.array([rng.integers(0, vocab)], np.int32)
        x = rng.standard_normal((1, hidden)).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
        qkv = rng.standard_normal((1, (nq + 2 * nkv) * hd)).astype(np.float32)
        qw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        kw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
        pos = np.array([rng.integers(0, 4096)], np.int32)
        g = rng.standard_normal((1, inter)).astype(np.float32)
        u = rng.standard_normal((1, inter)).astype(np.float32)

        # the reference: memcpy of the (fp32-converted) row, vDSP_vadd residual,
        # rmsnorm; per-head rmsnorm + apply_rope_cached on the model's table;
        # silu_vec_inplace(gate) * up
        e_ref = table[tok[0]].astype(np.float32)
        xs = (x[0] + e_ref).astype(np.float32)
        y_ref = np.empty(hidden, np.float32)
        ref.ref_rmsnorm(ptr(y_ref), ptr(xs), ptr(w), hidden, np.float32(1e-6))
        v = qkv[0, :(nq + nkv) * hd].copy().reshape(nq + nkv, hd)
        for h in range(nq + nkv):
            vh = np.ascontiguousarray(v[h])
            ref.ref_rmsnorm(ptr(vh), ptr(vh), ptr(qw if h < nq else kw), hd, np.float32(1e-6))
            v[h] = vh
        cs = np.empty(hd // 2, np.float32)
        sn = np.empty(hd // 2, np.float32)
        ref.ref_rope_row(ptr(cs), ptr(sn), int(pos[0]), hd, np.float32(1e6))
        v = np.ascontiguousarray(v)
        ref.ref_apply_rope_cached(ptr(v), C.c_void_p(v.ctypes.data + nq * hd * 4), nq, nkv, hd, hd,
                                  hd, hd, int(pos[0]), np.float32(1e6), ptr(cs), ptr(sn))
        sg = g[0].copy()
        ref.ref_silu_vec_inplace(ptr(sg), inter)
        h_ref = (sg * u[0]).astype(np.float32)

        tt = dev(table)
        e = ane.embedding_gather(tt, dev(tok), out_dtype=torch.float32)
        xt = dev(x)
        yt = ane.residual_rmsnorm(xt, e, dev(w))
        qt = dev(qkv)
        ane.qk_norm_rope(qt, dev(qw), dev(kw), dev(pos), nq, nkv, hd, theta=1e6)
        ht = ane.silu_mul(dev(g), dev(u))
        torch.cuda.synchronize()
        assert np.array_equal(e.cpu().numpy()[0].view(np.uint32), e_ref.view(np.uint32)), "gather"
        assert np.array_equal(xt.cpu().numpy()[0].view(np.uint32), xs.view(np.uint32)), "residual"
        for nm, got, want in (("rmsnorm", yt.cpu().numpy()[0], y_ref),
                              ("qk_norm_rope", qt.cpu().numpy()[0, :(nq + nkv) * hd], v.ravel()),
                              ("silu_mul", ht.cpu().numpy()[0], h_ref)):
            ok = within_2_f16_ulp(got, want)
            d32 = f32_ulp_diff(got, want)
            print(f"trial {trial} {nm}: max {int(d32.max())} fp32 ulp, "
                  f"{100 * float((d32 == 0).mean()):.2f}% bit-exact")
            assert ok.all(), (nm, int((~ok).sum()))


# --------------------------------------------------------------- golden fixtures
def test_rmsnorm_golden(ane):
    g = np.load(os.path.join(GOLDEN, "rmsnorm.npz"))
    for dim in (128, 1024, 2048, 4096, 1000):
        x, w, y = g[f"x_{dim}"], g[f"w_{dim}"], g[f"y_{dim}"]
        got = ane.residual_rmsnorm(dev(x), None, dev(w)).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), y.view(np.uint32)), dim


def test_qk_rope_golden(ane):
    """Per-head rmsnorm + RoPE against the reference's output with its libm
    table: the fused kernel (cos/sin in registers) within 2 fp16 ulp, and the
    table form (the golden cos/sin rows) bit-exact after the same norm."""
    g = np.load(os.path.join(GOLDEN, "qk_rope.npz"))
    nq, nkv, hd = (int(v) for v in g["shape"])
    qk_in, qk_out = g["qk_in"], g["qk_out"]
    rows = qk_in.shape[0]
    qkv = np.concatenate([qk_in.reshape(rows, -1), np.zeros((rows, nkv * hd), np.float32)], 1)
    qt = dev(qkv)
    ane.qk_norm_rope(qt, dev(g["qw"]), dev(g["kw"]), dev(g["positions"]), nq, nkv, hd,
                     theta=float(g["theta"]))
    got = qt.cpu().numpy()[:, :(nq + nkv) * hd].reshape(qk_out.shape)
    assert within_2_f16_ulp(got, qk_out).all()
    vmax = np.abs(qk_out).max()
    assert np.abs(got - qk_out).max() <= 4e-6 * vmax
    # table form: norm only (no RoPE: rot_dim 0), then apply_rope_cached on the table
    L = ane.lib()
    for i in range(rows):
        t = dev(np.ascontiguousarray(qkv[i:i + 1]))
        ane.qk_norm_rope(t, dev(g["qw"]), dev(g["kw"]), dev(g["positions"][i:i + 1]), nq, nkv, hd,
                         theta=float(g["theta"]), rot_dim=0)
        k = C.c_void_p(t.data_ptr() + nq * hd * 4)
        assert L.ane_cuda_apply_rope_cached(C.c_void_p(t.data_ptr()), k, nq, nkv, hd, hd, hd, hd,
                                            int(g["positions"][i]), float(g["theta"]),
                                            C.c_void_p(dev(g["cos"][i]).data_ptr()),
                                            C.c_void_p(dev(g["sin"][i]).data_ptr()), None) == 0
        _t().cuda.synchronize()
        got = t.cpu().numpy()[0, :(nq + nkv) * hd]
        assert np.array_equal(got.view(np.uint32), qk_out[i].ravel().view(np.uint32)), i


def test_silu_golden(ane):
    g = np.load(os.path.join(GOLDEN, "silu.npz"))
    t = dev(g["x"])
    assert ane.lib().ane_cuda_silu_inplace(0, C.c_void_p(t.data_ptr()), t.numel(), None) == 0
    _t().cuda.synchronize()
    assert np.array_equal(t.cpu().numpy().view(np.uint32), g["y"].view(np.uint32))


# --------------------------------------------------------------- sampler edge cases
def _edge_rows(vocab, rng):
    base = (rng.standard_normal(vocab) * 3).astype(np.float32)
    rows = {}

    def mk(name, f):
        a = base.copy()
        f(a)
        rows[name] = a

    mk("neg_inf_mask", lambda a: a.__setitem__(slice(0, vocab, 3), -np.inf))
    mk("pos_inf_one", lambda a: a.__setitem__(17, np.inf))
    mk("pos_inf_two", lambda a: (a.__setitem__(17, np.inf), a.__setitem__(vocab // 2, np.inf)))
    mk("nan_one", lambda a: a.__setitem__(40, np.nan))
    mk("nan_first", lambda a: a.__setitem__(0, np.nan))
    mk("nan_last", lambda a: a.__setitem__(vocab - 1, np.nan))
    mk("ties", lambda a: (a.__setitem__(10, 50.0), a.__setitem__(vocab - 20, 50.0)))
    mk("ties_at_zero", lambda a: (a.__setitem__(0, 60.0), a.__setitem__(5, 60.0)))
    mk("overflow_under_1_over_t", lambda a: a.__setitem__(33, 3e38))
    mk("all_but_one_neg_inf", lambda a: (a.fill(-np.inf), a.__setitem__(vocab // 3, 0.5)))
    rows["all_equal"] = np.full(vocab, 1.5, np.float32)
    rows["all_neg_inf"] = np.full(vocab, -np.inf, np.float32)
    rows["all_nan"] = np.full(vocab, np.nan, np.float32)
    return rows


@pytest.mark.parametrize("vocab", [1000, 151936])
def test_sampler_edge_cases_vs_reference(ane, ref, vocab):
    torch = _t()
    rng = np.random.default_rng(vocab + 1)
    rows = _edge_rows(vocab, rng)
    hist = rng.integers(0, vocab, 300).astype(np.int32)
    hist[:20] = 17  # penalise one of the +inf / special positions repeatedly
    names = list(rows)
    lg = np.stack([rows[n] for n in names])
    for temp in (0.6, 0.0):
        for use_hist in (False, True):
            want, us = [], []
            for i, n in enumerate(names):
                u = C.c_float()
                h = hist if use_hist else np.zeros(1, np.int32)
                t = ref.ref_sample_token(ptr(lg[i]), vocab, np.float32(temp), np.float32(1.2), 256,
                                         np.float32(0.1), ptr(h), h.size if use_hist else 0,
                                         500 + i, C.byref(u))
                want.append(t)
                us.append(u.value)
            hm = np.repeat(hist[None], len(names), 0) if use_hist else None
            hl = np.full(len(names), hist.size, np.int32) if use_hist else None
            got = ane.sample_rows(dev(lg), dev(np.array(us, np.float32)),
                                  None if hm is None else dev(hm), None if hl is None else dev(hl),
                                  temperature=temp).cpu().numpy()
            bad = [(n, int(g_), w_) for n, g_, w_ in zip(names, got, want) if g_ != w_]
            assert not bad, (temp, use_hist, bad)
    # uniforms at the edges: 0 (first element), NaN (never reached), 1.5 (past the end)
    row = np.stack([rows["ties"]] * 3)
    uu = np.array([0.0, np.nan, 1.5], np.float32)
    got = ane.sample_rows(dev(row), dev(uu), temperature=0.6).cpu().numpy()
    assert list(got) == [0, vocab - 1, vocab - 1]
    torch.cuda.synchronize()


@pytest.mark.parametrize("vocab", [1000, 151936])
def test_softmax_edge_rows_vs_reference(ane, ref, vocab):
    rng = np.random.default_rng(vocab + 2)
    rows = _edge_rows(vocab, rng)
    names = list(rows)
    lg = np.stack([rows[n] for n in names])
    got = ane.softmax_rows(dev(lg)).cpu().numpy()
    for i, n in enumerate(names):
        want = lg[i].copy()
        ref.ref_softmax(ptr(want), vocab)
        nan_w, nan_g = np.isnan(want), np.isnan(got[i])
        assert np.array_equal(nan_w, nan_g), n
        assert np.array_equal(got[i][~nan_g].view(np.uint32), want[~nan_w].view(np.uint32)), n


# --------------------------------------------------------------- RoPE fallback
def test_apply_rope_without_tables_vs_reference(ane, oracle, ref):
    L = ane.lib()
    rng = np.random.default_rng(8)
    for pos in (0, 1, 777, 4095, 100000):
        for rot, one_null in ((128, False), (64, False), (128, True)):
            q = rng.standard_normal((16, 128)).astype(np.float32)
            k = rng.standard_normal((8, 128)).astype(np.float32)
            qt, kt = dev(q), dev(k)
            table = dev(np.ones(64, np.float32))  # given alone, the reference ignores it
            st = L.ane_cuda_apply_rope_cached(C.c_void_p(qt.data_ptr()), C.c_void_p(kt.data_ptr()),
                                              16, 8, 128, 128, 128, rot, pos, 1e6,
                                              C.c_void_p(table.data_ptr()) if one_null else None,
                                              None, None)
            assert st == 0
            _t().cuda.synchronize()
            gq, gk = qt.cpu().numpy(), kt.cpu().numpy()
            oq, ok = oracle.apply_rope_interleaved(q, k, rot, pos, 1e6)
            assert np.array_equal(gq.view(np.uint32), oq.view(np.uint32))
            assert np.array_equal(gk.view(np.uint32), ok.view(np.uint32))
            rq, rk = q.copy(), k.copy()
            ref.ref_apply_rope_cached(ptr(rq), ptr(rk), 16, 8, 128, 128, 128, rot, pos,
                                      np.float32(1e6), None, None)
            vmax = max(np.abs(q).max(), np.abs(k).max())
            assert np.abs(gq - rq).max() <= 1e-6 * vmax and np.abs(gk - rk).max() <= 1e-6 * vmax
