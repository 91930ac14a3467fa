"""CPU tests of the oracle: the C restatement (oracle/oracle.c) against the
reference's own code compiled with the shim (oracle/_ref) and against the
committed golden fixtures that reference build produced."""
import ctypes as C
import os

import numpy as np
import pytest

from oracle_lib import F16, f16_ulp_diff, f32_ulp_diff

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def gold(name):
    return np.load(os.path.join(GOLDEN, name))


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- convert
def test_bf16_to_f16_golden_exhaustive(oracle):
    g = gold("bf16_to_f16.npz")
    assert np.array_equal(oracle.bf16_to_f16(g["bf16"]), g["f16"])


def test_bf16_to_f16_known_answers(oracle):
    # include/ane_lm/common.h:58-71 truncates and saturates NaN/overflow to Inf
    cases = {0x3F80: 0x3C00, 0x4780: 0x7C00, 0x7FC0: 0x7C00, 0x33C0: 0x0001, 0xFF80: 0xFC00,
             0x0000: 0x0000, 0x8000: 0x8000, 0x477F: 0x7BF8, 0x3380: 0x0001, 0x3300: 0x0000,
             0xC780: 0xFC00, 0x0001: 0x0000}
    inp = np.array(list(cases), np.uint16)
    got = oracle.bf16_to_f16(inp)
    assert [hex(v) for v in got] == [hex(v) for v in cases.values()]


# ---------------------------------------------------------------- pinned math
def test_expf_accuracy(oracle):
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.uniform(-104, 88.7, 100000), rng.uniform(-1, 1, 20000),
                        [0.0, -0.0, 1.0, -1.0, 88.7, -87.3]]).astype(np.float32)
    e = oracle.expf(x)
    t = np.exp(x.astype(np.float64)).astype(np.float32)
    normal = t > np.float32(1.2e-38)
    assert f32_ulp_diff(e[normal], t[normal]).max() <= 1
    assert np.all(np.abs(e[~normal] - t[~normal]) <= np.float32(2 ** -149))
    assert oracle.expf(np.array([0.0], np.float32))[0] == 1.0
    assert oracle.expf(np.array([-105.0], np.float32))[0] == 0.0
    assert np.isinf(oracle.expf(np.array([89.0], np.float32))[0])


def test_sincos_accuracy(oracle):
    rng = np.random.default_rng(4)
    xs = np.concatenate([rng.uniform(0, 4096, 5000), rng.uniform(0, 2e5, 2000),
                         [0.0, 1e-8, np.pi / 4, np.pi / 2, 100000.0]]).astype(np.float32)
    worst = 0
    for v in xs:
        s, c = oracle.sincosf(v)
        ts = np.float32(np.sin(np.float64(v)))
        tc = np.float32(np.cos(np.float64(v)))
        # absolute error relative to 1 ulp at magnitude 1 keeps near-zero values fair
        worst = max(worst, abs(s - ts) / 2 ** -24, abs(c - tc) / 2 ** -24)
    assert worst <= 2.0


def test_rope_inv_freq_matches_model_table(oracle, ref):
    # models/llm/qwen3.cpp:205-208 with libm powf vs the oracle's rounded double pow
    inv = oracle.rope_inv_freq(128, 1e6)
    cos = np.empty(64, np.float32)
    sin = np.empty(64, np.float32)
    ref.ref_rope_row(ptr(cos), ptr(sin), 1, 128, np.float32(1e6))
    # at pos = 1 the reference's angle is exactly inv_freq
    for j in range(64):
        s, c = oracle.sincosf(inv[j])
        assert abs(c - cos[j]) <= 2 ** -23 and abs(s - sin[j]) <= 2 ** -23


def test_rope_fallback_matches_reference(oracle, ref):
    """apply_rope_cached without tables takes the reference's fallback over
    interleaved pairs with libm powf / cosf / sinf (core/cpu_ops.cpp:66-77);
    the restatement (pinned inv_freq and sincos) stays within 1e-6 x max|v|
    of the reference build, at positions 0 .. 2^20 and two rotary widths."""
    import ctypes as C
    rng = np.random.default_rng(21)
    for pos in (0, 1, 2, 7, 100, 777, 2047, 4095, 16383, 100000, 1 << 20):
        for rot in (128, 64):
            q = rng.standard_normal((16, 128)).astype(np.float32)
            k = rng.standard_normal((8, 128)).astype(np.float32)
            oq, ok = oracle.apply_rope_interleaved(q, k, rot, pos, 1e6)
            rq, rk = q.copy(), k.copy()
            ref.ref_apply_rope_cached(ptr(rq), ptr(rk), 16, 8, 128, 128, 128, rot, pos,
                                      np.float32(1e6), None, None)
            vmax = max(np.abs(q).max(), np.abs(k).max())
            assert np.abs(oq - rq).max() <= 1e-6 * vmax and np.abs(ok - rk).max() <= 1e-6 * vmax
            # elements past rot_dim are untouched
            assert np.array_equal(oq[:, rot:], q[:, rot:]) and np.array_equal(rq[:, rot:], q[:, rot:])


# ---------------------------------------------------------------- rmsnorm
def test_rmsnorm_f32_golden(oracle):
    g = gold("rmsnorm.npz")
    for dim in (128, 1024, 2048, 4096, 1000):
        x, w, y = g[f"x_{dim}"], g[f"w_{dim}"], g[f"y_{dim}"]
        _, got = oracle.residual_rmsnorm(x, None, w)
        # the shim's vDSP_svesq is the pinned 32-lane order over 4-float chunks,
        # so the fp32 restatement is bit-exact with the reference routine
        assert np.array_equal(got, y), dim


def test_rmsnorm_f16_vs_reference(oracle, ref):
    rng = np.random.default_rng(5)
    for dim in (1024, 2048, 4096):
        x = rng.standard_normal((8, dim)).astype(np.float16)
        d = rng.standard_normal((8, dim)).astype(np.float16)
        w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        xo, yo = oracle.residual_rmsnorm(x, d, w)
        xs = (x.astype(np.float32) + d.astype(np.float32)).astype(np.float16)
        assert np.array_equal(xo, xs)
        yr = np.empty((8, dim), np.float32)
        xf = xs.astype(np.float32)
        for r in range(8):
            ref.ref_rmsnorm(ptr(yr[r]), ptr(xf[r]), ptr(w), dim, np.float32(1e-6))
        assert f16_ulp_diff(yo, yr.astype(np.float16)).max() <= 1


# ---------------------------------------------------------------- QK-norm + RoPE
def test_qk_norm_rope_golden(oracle):
    g = gold("qk_rope.npz")
    nq, nkv, hd = (int(v) for v in g["shape"])
    qk_in = g["qk_in"]
    rows = qk_in.shape[0]
    qkv = np.concatenate([qk_in.reshape(rows, -1), np.zeros((rows, nkv * hd), np.float32)], 1)
    got = oracle.qk_norm_rope(qkv, nq, nkv, hd, g["qw"], g["kw"], g["positions"],
                              float(g["theta"]))
    got = got[:, :(nq + nkv) * hd].reshape(qk_in.shape)
    want = g["qk_out"]
    # the reference table uses libm cosf/sinf, the oracle its pinned sin/cos;
    # both are within ~1 ulp of the true values
    scale = np.maximum(np.abs(want), 1.0)
    assert np.max(np.abs(got - want) / scale) < 2e-6
    assert f16_ulp_diff(got.astype(np.float16), want.astype(np.float16)).max() <= 1


# ---------------------------------------------------------------- SiLU
def test_silu_golden(oracle):
    g = gold("silu.npz")
    x = g["x"][None, :]
    got = oracle.silu_mul(x, np.ones_like(x))[0]
    # vvexpf is the pinned exp in both: bit-exact
    assert np.array_equal(got.view(np.int32), g["y"].view(np.int32))


# ---------------------------------------------------------------- sampler
def test_sampler_golden(oracle):
    g = gold("sampler.npz")
    for i in range(g["tokens"].size):
        tok = oracle.sample_rows(g["logits"][i:i + 1], g["uniforms"][i:i + 1],
                                 g["history"][i:i + 1], g["history_len"][i:i + 1],
                                 temperature=float(g["temperature"][i]), rep=float(g["rep"][i]))
        assert tok[0] == g["tokens"][i], i


@pytest.mark.parametrize("vocab", [7, 1000, 151936])
def test_sampler_vs_reference(oracle, ref, vocab):
    rng = np.random.default_rng(vocab)
    n = 6 if vocab > 100000 else 40
    for i in range(n):
        lg = (rng.standard_normal(vocab) * 3).astype(np.float32)
        hl = int(rng.integers(0, 1100))
        hist = rng.integers(-2, vocab + 2, size=max(hl, 1)).astype(np.int32)
        temp = [0.6, 0.0, 1.3, -1.0][i % 4]
        u = C.c_float()
        want = ref.ref_sample_token(ptr(lg), vocab, np.float32(temp), np.float32(1.2), 256,
                                    np.float32(0.1), ptr(hist), hl, 77 + i, C.byref(u))
        got = oracle.sample_rows(lg[None], np.array([u.value], np.float32), hist[None],
                                 np.array([hl], np.int32), temperature=temp)
        assert got[0] == want, (i, temp, hl)


# ---------------------------------------------------------------- gather
def test_gather(oracle):
    rng = np.random.default_rng(9)
    table = rng.standard_normal((100, 64)).astype(np.float16)
    ids = np.array([0, 99, 5, -1, 100, 42], np.int32)
    out, bad = oracle.embedding_gather(table, ids)
    assert bad == 2
    assert np.array_equal(out[[0, 1, 2, 5]], table[[0, 99, 5, 42]])
    assert not out[[3, 4]].any()
    out32, _ = oracle.embedding_gather(table, ids, out_dtype=0)
    assert np.array_equal(out32[0], table[0].astype(np.float32))


# ---------------------------------------------------------------- whole chain
def test_layer_chain_f16_vs_reference(oracle, ref):
    rng = np.random.default_rng(11)
    rows, hidden, nq, nkv, hd, inter = 6, 512, 4, 2, 128, 768
    x = rng.standard_normal((rows, hidden)).astype(np.float16)
    d = rng.standard_normal((rows, hidden)).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    qkv = rng.standard_normal((rows, (nq + 2 * nkv) * hd)).astype(np.float16)
    qw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    pos = np.array([0, 1, 5, 511, 2047, 9000], np.int32)
    g = rng.standard_normal((rows, inter)).astype(np.float16)
    u = rng.standard_normal((rows, inter)).astype(np.float16)
    g[0, :5] *= 50

    xr, yr, qr, hr = x.copy(), np.empty_like(x), qkv.copy(), np.empty_like(g)
    ref.ref_layer_chain_f16(ptr(xr), ptr(d), ptr(yr), ptr(w), ptr(qr), ptr(qw), ptr(kw), ptr(pos),
                            ptr(g), ptr(u), ptr(hr), 0, rows, hidden, nq, nkv, hd, inter,
                            np.float32(1e6), np.float32(1e-6))
    xo, yo = oracle.residual_rmsnorm(x, d, w)
    qo = oracle.qk_norm_rope(qkv, nq, nkv, hd, qw, kw, pos, 1e6)
    ho = oracle.silu_mul(g, u)
    assert np.array_equal(xo, xr)
    assert f16_ulp_diff(yo, yr).max() <= 2
    assert f16_ulp_diff(qo, qr).max() <= 2
    assert f16_ulp_diff(ho, hr).max() <= 2


# ---------------------------------------------------------- decode attention
@pytest.mark.parametrize("H,hk,hd,cap,start,ln", [
    (16, 8, 128, 4096, 1000, 4096), (32, 8, 128, 300, 250, 290), (16, 8, 128, 512, 7, 1),
    (8, 8, 64, 100, 99, 37), (16, 2, 256, 129, 5, 129), (16, 8, 128, 64, 0, 0)])
def test_attention_oracle_vs_reference(oracle, ref, H, hk, hd, cap, start, ln):
    """The pinned split order stays within 1e-6 x max|v| of the reference's
    sequential sums (core/cpu_ops.cpp:173-240 with the shim)."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal((1, H, hd)).astype(np.float32)
    k = rng.standard_normal((1, cap, hk, hd)).astype(np.float32)
    v = rng.standard_normal((1, cap, hk, hd)).astype(np.float32)
    got = oracle.decode_attention(q, k, v, [start], [ln])[0]
    want = np.empty((H, hd), np.float32)
    ref.ref_gqa_attention(ptr(want), ptr(q), ptr(k), ptr(v), H, hk, hd, hd, start, ln, cap)
    assert np.abs(got - want).max() <= 1e-6 * np.abs(v).max()
    if ln == 0:
        assert not np.any(got) and not np.any(want)


def test_attention_oracle_half_types(oracle):
    """fp16 caches: the fp32 arithmetic on the widened values, rounded once
    at the end.  (head_dim 256: 8 elements per lane for both element sizes,
    so fp16 and fp32 take the same summation order.)"""
    rng = np.random.default_rng(4)
    q = rng.standard_normal((1, 16, 256)).astype(np.float16)
    k = rng.standard_normal((1, 200, 8, 256)).astype(np.float16)
    v = rng.standard_normal((1, 200, 8, 256)).astype(np.float16)
    o16 = oracle.decode_attention(q, k, v, [150], [200])
    o32 = oracle.decode_attention(q.astype(np.float32), k.astype(np.float32),
                                  v.astype(np.float32), [150], [200])
    assert np.array_equal(o16, o32.astype(np.float16))


def test_kv_ring_advance():
    """models/llm/qwen3.cpp:475-484: fill, then overwrite the oldest slot."""
    from oracle_lib import Oracle
    o = Oracle()
    start, ln, cap = 0, 0, 4
    slots = []
    for _ in range(7):
        slot, start, ln = o.kv_ring_advance(start, ln, cap)
        slots.append(slot)
    assert slots == [0, 1, 2, 3, 0, 1, 2]
    assert (start, ln) == (3, 4)


# ------------------------------------------- fp32 <-> fp16 at the ANE boundary
def _f32_samples(n=1 << 20):
    rng = np.random.default_rng(21)
    bits = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    special = np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00001, 0x7F800001,
                        0x33000000, 0x33000001, 0x387FC000, 0x38800000, 0x477FE000, 0x477FF000,
                        0x477FEFFF, 0x00000001, 0x807FFFFF, 0x3F800000, 0x3F801000, 0x3F803000],
                       np.uint32)
    vals = (rng.standard_normal(n).astype(np.float32) * np.float32(100)).view(np.uint32)
    return np.concatenate([special, bits, vals]).view(np.float32)


def test_f32_to_f16_trunc_vs_reference(oracle, ref):
    """The x86 packing conversion: bit-exact against the reference's
    f32_to_f16 (include/ane_lm/common.h:58-71) over random bit patterns."""
    x = _f32_samples()
    want = np.empty(x.size, np.uint16)
    ref.ref_f32_to_f16_vec(ptr(want), ptr(x), x.size)
    got = oracle.ane_pack(x.reshape(1, -1), round_mode=1, spatial=1).ravel()
    assert np.array_equal(got, want)


def test_f32_to_f16_rne_vs_numpy(oracle):
    """The arm64 packing conversion is IEEE round-to-nearest-even (numpy's
    float32 -> float16); NaN becomes the quiet NaN 0x7E00 with its sign."""
    x = _f32_samples()
    got = oracle.ane_pack(x.reshape(1, -1), round_mode=0, spatial=1).ravel()
    nan = np.isnan(x)
    with np.errstate(over="ignore", invalid="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got[~nan], want[~nan])
    sign = (x.view(np.uint32)[nan] >> 16) & 0x8000
    assert np.array_equal(got[nan], (0x7E00 | sign).astype(np.uint16))


def test_f16_to_f32_vs_reference(oracle, ref):
    """Unpacking widens exactly: all 65,536 halves, NaN payloads included,
    bit-exact against the reference's f16_to_f32."""
    h = np.arange(1 << 16, dtype=np.uint16)
    want = np.empty(h.size, np.float32)
    ref.ref_f16_to_f32_vec(ptr(want), ptr(h), h.size)
    got = oracle.ane_unpack(h.reshape(1, -1, 1), tokens=1, spatial=1).ravel()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_ane_pack_layout(oracle):
    """Token t -> surface t // 32, spatial slot t % 32, channel stride 32;
    other slots keep their contents; unpack inverts pack on fp16 values."""
    rng = np.random.default_rng(22)
    t, c = 45, 7
    x = rng.standard_normal((t, c)).astype(np.float16).astype(np.float32)
    base = np.full((2, c, 32), 0xABCD, np.uint16)
    s = oracle.ane_pack(x, surface=base)
    assert s.shape == (2, c, 32)
    assert np.array_equal(s[1, :, 13:], base[1, :, 13:])
    assert np.array_equal(s[1, 3, 12], x[44, 3].astype(np.float16).view(np.uint16))
    assert np.array_equal(s[0, 5, 31], x[31, 5].astype(np.float16).view(np.uint16))
    assert np.array_equal(oracle.ane_unpack(s, t), x)


# ------------------------------------------------------ hybrid-model row ops
@pytest.mark.parametrize("dim", [128, 64, 100])
def test_rmsnorm_gated_vs_reference(oracle, ref, dim):
    """rmsnorm_gated (core/cpu_ops.cpp:33-39): bit-exact, fp32."""
    rng = np.random.default_rng(dim)
    rows = 6
    x = rng.standard_normal((rows, dim)).astype(np.float32) * 3
    z = rng.standard_normal((rows, dim)).astype(np.float32) * 4
    z[0, :4] = [-90.0, 90.0, -0.0, 40.0]
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    got = oracle.rmsnorm_gated(x, z, w)
    for r in range(rows):
        want = np.empty(dim, np.float32)
        ref.ref_rmsnorm_gated(ptr(want), ptr(x[r]), ptr(z[r]), ptr(w), dim)
        assert np.array_equal(got[r].view(np.uint32), want.view(np.uint32)), r


@pytest.mark.parametrize("dim", [128, 64, 100, 4096])
def test_l2_normalize_vs_reference(oracle, ref, dim):
    """l2_normalize (core/cpu_ops.cpp:106-111): bit-exact, fp32, a zero row too."""
    rng = np.random.default_rng(dim + 1)
    x = rng.standard_normal((5, dim)).astype(np.float32) * 2
    x[3] = 0.0
    got = oracle.l2_normalize(x)
    for r in range(5):
        want = x[r].copy()
        ref.ref_l2_normalize(ptr(want), dim)
        assert np.array_equal(got[r].view(np.uint32), want.view(np.uint32)), r


def test_norm_weight_load_vs_reference(oracle, ref, tmp_path):
    """load_bf16_to_f32 and the (1 + w) load_norm_weight (core/safetensors.cpp:
    264-306) of a BF16 tensor: bit-exact, specials included."""
    from safetensors_util import write_safetensors
    rng = np.random.default_rng(9)
    b = rng.integers(0, 1 << 16, 4096, dtype=np.uint64).astype(np.uint16)
    b[:6] = [0x0000, 0x8000, 0x7F80, 0xFF80, 0x7FC0, 0x3F80]
    path = str(tmp_path / "w.safetensors")
    write_safetensors(path, [("model.norm.weight", "BF16", b)])
    for norm in (0, 1):
        want = np.empty(4096, np.float32)
        assert ref.ref_load_weight(path.encode(), b"model.norm.weight", 4096, norm, ptr(want)) == 0
        got = oracle.bf16_to_f32_weights(b, norm)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), norm


# ------------------------------------------- golden fixtures of the next rows
def test_gqa_attention_golden(oracle):
    """The oracle's attention within 1e-6 x max|v| of the reference's outputs
    in tests/golden/gqa_attention.npz (different, fixed summation orders)."""
    g = np.load(os.path.join(GOLDEN, "gqa_attention.npz"))
    i = 0
    while f"q{i}" in g:
        q, k, v = (g[f"{n}{i}"].astype(np.float32) for n in "qkv")
        start, ln, cap = (int(t) for t in g[f"ring{i}"])
        got = oracle.decode_attention(q[None], k[None], v[None], [start], [ln])[0]
        assert np.abs(got - g[f"out{i}"]).max() <= 1e-6 * np.abs(v).max(), i
        i += 1
    assert i == 5


def test_hybrid_rows_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "hybrid_rows.npz"))
    gated = oracle.rmsnorm_gated(g["x"], g["z"], g["w"])
    assert np.array_equal(gated.view(np.uint32), g["gated"].view(np.uint32))
    l2 = oracle.l2_normalize(g["x"])
    assert np.array_equal(l2.view(np.uint32), g["l2"].view(np.uint32))


def test_ane_convert_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "ane_convert.npz"))
    got = oracle.ane_pack(g["f32"].reshape(1, -1), round_mode=1, spatial=1).ravel()
    assert np.array_equal(got, g["trunc"])
    h = np.arange(65536, dtype=np.uint16)
    w = oracle.ane_unpack(h.reshape(1, -1, 1), tokens=1, spatial=1).ravel()
    assert np.array_equal(w.view(np.uint32), g["widen"].view(np.uint32))


def test_norm_weight_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "norm_weight.npz"))
    for key, add in (("plain", False), ("norm", True)):
        got = oracle.bf16_to_f32_weights(g["bf16"], add)
        assert np.array_equal(got.view(np.uint32), g[key].view(np.uint32)), key
