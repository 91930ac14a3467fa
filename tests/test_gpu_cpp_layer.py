"""GPU: the reference-signature C++ layer (ane-lm_b200/core/cuda_ops.h), driven
by a C++ program compiled here against the library, checked against the
oracle -- the path a maintainer takes when dropping it into ANE-LM."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest


pytestmark = pytest.mark.gpu
TESTS = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(TESTS)
PKG = os.path.join(REPO, "ane-lm_b200")
CUDA = "/usr/local/cuda"


def drand48_floats(seed, n):
    """(float)drand48() after srand48(seed): the POSIX 48-bit LCG."""
    x = ((seed & 0xFFFFFFFF) << 16) | 0x330E
    out = []
    for _ in range(n):
        x = (0x5DEECE66D * x + 0xB) & ((1 << 48) - 1)
        out.append(np.float32(x / float(1 << 48)))
    return np.array(out, np.float32)


@pytest.fixture(scope="module")
def checker(ane, tmp_path_factory):
    d = tmp_path_factory.mktemp("cpp")
    exe = str(d / "cuda_ops_check")
    subprocess.run(["g++", "-O2", "-std=c++17", os.path.join(TESTS, "cpp", "cuda_ops_check.cpp"),
                    "-I", os.path.join(REPO, "include"), "-I", os.path.join(PKG, "core"),
                    "-I", f"{CUDA}/include", "-L", PKG, "-lane_cuda", "-L", f"{CUDA}/lib64",
                    "-lcudart", f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{CUDA}/lib64", "-o", exe],
                   check=True)
    return exe, d


def test_reference_signature_layer(checker, oracle):
    exe, d = checker
    rng = np.random.default_rng(7)
    dim, hd, nq, nkv, n, vocab = 2048, 128, 16, 8, 3072, 151936
    x = rng.standard_normal(dim).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    qk = rng.standard_normal((nq + nkv) * hd).astype(np.float32)
    cosr = np.cos(rng.uniform(0, 6, hd // 2)).astype(np.float32)
    sinr = np.sin(rng.uniform(0, 6, hd // 2)).astype(np.float32)
    g = (rng.standard_normal(n) * 4).astype(np.float32)
    z = (rng.standard_normal(n) * 4).astype(np.float32)
    logits = (rng.standard_normal(vocab) * 3).astype(np.float32)
    hist = rng.integers(0, vocab, 300).astype(np.int32)
    bf = rng.integers(0, 65536, 1000).astype(np.uint16)
    cap = 300
    kc = rng.standard_normal((cap, nkv, hd)).astype(np.float32)
    vc = rng.standard_normal((cap, nkv, hd)).astype(np.float32)
    inp, outp = d / "in.bin", d / "out.bin"
    with open(inp, "wb") as f:
        for a in (x, w, qk, cosr, sinr, g, z, logits, hist, bf, kc, vc):
            f.write(a.tobytes())
    subprocess.run([exe, str(inp), str(outp)], check=True, timeout=120)
    raw = outp.read_bytes()
    off = 0

    def take(dtype, count):
        nonlocal off
        a = np.frombuffer(raw, dtype, count, off)
        off += a.nbytes
        return a

    # rmsnorm in place: bit-exact with the oracle's fp32 rmsnorm
    _, y = oracle.residual_rmsnorm(x[None], None, w)
    assert np.array_equal(take(np.float32, dim), y[0])
    # apply_rope_cached with caller tables: v0' = v0 c - v1 s, v1' = v1 c + v0 s
    heads = qk.reshape(-1, hd)
    a0, a1 = heads[:, :hd // 2], heads[:, hd // 2:]
    want = np.concatenate([a0 * cosr - a1 * sinr, a1 * cosr + a0 * sinr], 1).ravel()
    assert np.array_equal(take(np.float32, qk.size), want)
    # no tables: the reference's fallback over interleaved pairs
    # (core/cpu_ops.cpp:66-77), cos/sin of the pinned sincos in registers
    nh = heads.shape[0]
    wq, wk = oracle.apply_rope_interleaved(heads[:nq], heads[nq:], hd, 777, 1e6)
    want = np.concatenate([wq, wk]).ravel()
    assert nh == nq + nkv
    assert np.array_equal(take(np.float32, qk.size), want)
    # silu_vec_inplace / mul_sigmoid_inplace (fp32: pinned exp, IEEE divide)
    assert np.array_equal(take(np.float32, n), oracle.silu_mul(g[None], np.ones((1, n), np.float32))[0])
    e = oracle.expf(-z)
    assert np.array_equal(take(np.float32, n), g / (np.float32(1) + e))
    # softmax
    assert np.array_equal(take(np.float32, vocab), oracle.softmax_rows(logits[None])[0])
    # sample_token: srand48(4242); four draws, greedy (no draw), one draw without history
    u = drand48_floats(4242, 5)
    toks = take(np.int32, 6)
    for i in range(4):
        assert toks[i] == oracle.sample_rows(logits[None], u[i:i + 1], hist[None],
                                             np.array([300], np.int32))[0]
    assert toks[4] == oracle.sample_rows(logits[None], u[:1], hist[None], np.array([300], np.int32),
                                         temperature=0.0)[0]
    assert toks[5] == oracle.sample_rows(logits[None], u[4:5])[0]
    # bf16_to_f16_vec
    assert np.array_equal(take(np.uint16, bf.size), oracle.bf16_to_f16(bf))
    # rmsnorm_gated per head (x as 16 heads of 128, z's first 2048, w's first 128)
    want = oracle.rmsnorm_gated(x.reshape(-1, hd), z[:dim].reshape(-1, hd), w[:hd]).ravel()
    assert np.array_equal(take(np.float32, dim), want)
    # l2_normalize per head of qk
    assert np.array_equal(take(np.float32, qk.size), oracle.l2_normalize(qk.reshape(-1, hd)).ravel())
    # gqa_attention: q = the first 16 heads of qk, ring start 250, 290 keys of 300
    q = qk[:nq * hd].reshape(1, nq, hd)
    want = oracle.decode_attention(q, kc[None], vc[None], [250], [290])[0].ravel()
    assert np.array_equal(take(np.float32, nq * hd), want)
    assert not np.any(take(np.float32, nq * hd))
    # kv_ring_advance: the reference's ring (fill, then overwrite the oldest)
    want = []
    st_, ln_ = 0, 0
    for _ in range(7):
        slot, st_, ln_ = oracle.kv_ring_advance(st_, ln_, 4)
        want.append(slot)
    assert list(take(np.int32, 9)) == want + [st_, ln_]
    # a failing call reports through last_status() and the process carries on
    assert take(np.int32, 1)[0] == 1
    assert off == len(raw)


def test_sample_token_decode_loop(ane, ref, tmp_path):
    """1,000 decode steps through the drop-in sample_token with a growing
    history (Qwen3 vocabulary, T 0.6, penalty 1.2 over the last 256 ids,
    frequency 0.1): every token equals the reference's own loop with the
    same srand48 seed, and the device's free memory does not change after
    the first call (the staging is fixed: only the window is copied)."""
    exe = str(tmp_path / "sample_loop")
    subprocess.run(["g++", "-O2", "-std=c++17", os.path.join(TESTS, "cpp", "sample_loop.cpp"),
                    "-I", os.path.join(REPO, "include"), "-I", os.path.join(PKG, "core"),
                    "-I", f"{CUDA}/include", "-L", PKG, "-lane_cuda", "-L", f"{CUDA}/lib64",
                    "-lcudart", f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{CUDA}/lib64", "-o", exe],
                   check=True)
    rng = np.random.default_rng(99)
    nrows, vocab, ctx, steps, seed = 8, 151936, 256, 1000, 4321
    logits = (rng.standard_normal((nrows, vocab)) * 3).astype(np.float32)
    # a peaked row or two, so the history repeats ids and the penalties bite
    logits[3, 5:9] += 30.0
    hist0 = rng.integers(0, vocab, 100).astype(np.int32)
    temp, rep, freq = 0.6, 1.2, 0.1
    inp, outp = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(inp, "wb") as f:
        f.write(np.array([nrows, vocab, ctx, hist0.size, steps, seed], np.int32).tobytes())
        f.write(np.array([temp, rep, freq], np.float32).tobytes())
        f.write(logits.tobytes())
        f.write(hist0.tobytes())
    subprocess.run([exe, str(inp), str(outp)], check=True, timeout=300)
    raw = outp.read_bytes()
    got = np.frombuffer(raw, np.int32, steps)
    mem = np.frombuffer(raw, np.int64, 2, steps * 4)
    want = np.empty(steps, np.int32)
    ref.ref_sample_token_loop(logits.ctypes.data_as(C.c_void_p), nrows, vocab, np.float32(temp),
                              np.float32(rep), ctx, np.float32(freq),
                              hist0.ctypes.data_as(C.c_void_p), hist0.size, seed, steps,
                              want.ctypes.data_as(C.c_void_p))
    assert np.array_equal(got, want), int(np.argmax(got != want))
    assert len(set(want.tolist())) < steps  # repeats: the penalties were exercised
    assert mem[0] == mem[1], mem
