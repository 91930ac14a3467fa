"""GPU parity of the sampler and softmax: token ids bit-exact against the
oracle (itself bit-exact against the reference's sample_token) given the
same logits and uniforms."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _torch():
    import torch
    return torch


def dev(a):
    return _torch().from_numpy(np.ascontiguousarray(a)).cuda()


def run(ane, logits, u, hist=None, hlen=None, **kw):
    out = ane.sample_rows(dev(logits), dev(u), None if hist is None else dev(hist),
                          None if hlen is None else dev(hlen), **kw)
    return out.cpu().numpy()


def test_sampler_golden(ane):
    g = np.load(os.path.join(GOLDEN, "sampler.npz"))
    for i in range(g["tokens"].size):
        got = run(ane, g["logits"][i:i + 1], g["uniforms"][i:i + 1], g["history"][i:i + 1],
                  g["history_len"][i:i + 1], temperature=float(g["temperature"][i]),
                  repetition_penalty=float(g["rep"][i]))
        assert got[0] == g["tokens"][i], i


def test_sampler_config4_batch256(ane, oracle):
    """256 x 151936, logits N(0,3), 1024-id histories."""
    rng = np.random.default_rng(4)
    rows, vocab = 256, 151936
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    hist = rng.integers(0, vocab, size=(rows, 1024)).astype(np.int32)
    hlen = np.full(rows, 1024, np.int32)
    u = rng.random(rows).astype(np.float32)
    got = run(ane, logits, u, hist, hlen, temperature=0.6)
    want = oracle.sample_rows(logits, u, hist, hlen, temperature=0.6)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:10]


def test_sampler_cta_size_does_not_change_tokens(ane, oracle):
    """A batch of at most one row per SM runs 1024-thread CTAs, a larger one
    512-thread CTAs; both keep the 1024-virtual-thread orders, so the same
    rows give the same tokens alone (small batch) and inside a batch of 300
    (more rows than SMs), all equal to the oracle's.  Greedy rows included."""
    rng = np.random.default_rng(45)
    rows, vocab = 300, 151936
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    hist = rng.integers(0, vocab, size=(rows, 1024)).astype(np.int32)
    hlen = rng.integers(0, 1025, size=rows).astype(np.int32)
    u = rng.random(rows).astype(np.float32)
    u[:4] = (0.0, np.float32(0.99999994), 0.5, 0.999)
    for temp in (0.6, 0.0):
        big = run(ane, logits, u, hist, hlen, temperature=temp)
        want = oracle.sample_rows(logits, u, hist, hlen, temperature=temp)
        assert np.array_equal(big, want), (temp, np.nonzero(big != want)[0][:10])
        for r0, n in ((0, 1), (5, 32), (40, 100), (150, 148)):
            small = run(ane, logits[r0:r0 + n], u[r0:r0 + n], hist[r0:r0 + n], hlen[r0:r0 + n],
                        temperature=temp)
            assert np.array_equal(small, want[r0:r0 + n]), (temp, r0, n)


@pytest.mark.parametrize("vocab", [1, 3, 7, 64, 1001, 4096, 32000, 151936])
def test_sampler_vocab_sizes(ane, oracle, vocab):
    rng = np.random.default_rng(vocab)
    rows = 24
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    hist = rng.integers(-5, vocab + 5, size=(rows, 300)).astype(np.int32)
    hlen = rng.integers(0, 301, size=rows).astype(np.int32)
    u = rng.random(rows).astype(np.float32)
    u[0], u[1] = 0.0, np.float32(0.99999994)
    for temp in (0.6, 0.0, 1.7):
        got = run(ane, logits, u, hist, hlen, temperature=temp)
        want = oracle.sample_rows(logits, u, hist, hlen, temperature=temp)
        assert np.array_equal(got, want), (temp, np.nonzero(got != want)[0][:10])


@pytest.mark.parametrize("base", [-1000.0, -20.0, 0.0, 25.0, 1000.0])
def test_sampler_offsets_scales_temperatures(ane, oracle, base):
    """The CDF scan tests logits against a floor derived from the binade's
    significance threshold (d = fl(fl(v / T) - max)): offsets that make the
    max large, near zero or negative, spreads from flat to peaked, and
    temperatures from cold to hot, with every u from 0 to just below 1."""
    rng = np.random.default_rng(int(base) + 5000)
    vocab, rows = 20000, 12
    for sigma in (0.05, 3.0, 80.0):
        logits = (base + rng.standard_normal((rows, vocab)) * sigma).astype(np.float32)
        u = np.linspace(0, 0.99999994, rows).astype(np.float32)
        for temp in (0.05, 0.6, 3.0):
            got = run(ane, logits, u, temperature=temp, repetition_penalty=1.0)
            want = oracle.sample_rows(logits, u, temperature=temp, rep=1.0)
            assert np.array_equal(got, want), (sigma, temp, np.nonzero(got != want)[0][:10])


def test_sampler_edge_distributions(ane, oracle):
    vocab = 50000
    rows = []
    rows.append(np.zeros(vocab, np.float32))                         # uniform
    r = np.full(vocab, -30.0, np.float32); r[12345] = 30.0; rows.append(r)  # one-hot
    r = np.full(vocab, -1e30, np.float32); r[-1] = 0.0; rows.append(r)      # mass at the end
    r = np.linspace(-20, 20, vocab).astype(np.float32); rows.append(r)      # rising
    r = np.linspace(20, -20, vocab).astype(np.float32); rows.append(r)      # falling
    rng = np.random.default_rng(8)
    rows.append((rng.standard_normal(vocab) * 30).astype(np.float32))       # very peaked
    rows.append((rng.standard_normal(vocab) * 0.01).astype(np.float32))     # nearly flat
    logits = np.stack(rows)
    for seed in range(6):
        u = np.random.default_rng(seed).random(len(rows)).astype(np.float32)
        for temp in (0.6, 1.0, 0.05):
            got = run(ane, logits, u, temperature=temp)
            want = oracle.sample_rows(logits, u, temperature=temp)
            assert np.array_equal(got, want), (seed, temp, got, want)


def test_sampler_penalty_paths(ane, oracle):
    rng = np.random.default_rng(12)
    vocab, rows = 2000, 16
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    hist = rng.integers(0, 40, size=(rows, 600)).astype(np.int32)  # heavy repeats
    hlen = np.full(rows, 600, np.int32)
    u = rng.random(rows).astype(np.float32)
    for rep, freq, ctx in [(1.2, 0.1, 256), (1.0, 0.1, 256), (1.5, 0.0, 600), (1.2, 0.3, 0),
                           (1.2, 0.1, 4096), (0.5, 0.1, 10)]:
        got = run(ane, logits, u, hist, hlen, temperature=0.6, repetition_penalty=rep,
                  frequency_penalty=freq, repetition_context=ctx)
        want = oracle.sample_rows(logits, u, hist, hlen, temperature=0.6, rep=rep, ctx=ctx,
                                  freq=freq)
        assert np.array_equal(got, want), (rep, freq, ctx)
    # greedy with penalties
    got = run(ane, logits, u, hist, hlen, temperature=0.0)
    want = oracle.sample_rows(logits, u, hist, hlen, temperature=0.0)
    assert np.array_equal(got, want)


def test_sampler_many_seeds_full_vocab(ane, oracle):
    """A few thousand (row, u) draws at the full vocabulary: exercises the
    binade crossings and the serial fallback of the parallel CDF scan."""
    rng = np.random.default_rng(99)
    vocab, rows = 151936, 64
    logits = (rng.standard_normal((rows, vocab)) * 3).astype(np.float32)
    for k in range(8):
        u = rng.random(rows).astype(np.float32)
        got = run(ane, logits, u, temperature=0.6)
        want = oracle.sample_rows(logits, u, temperature=0.6)
        assert np.array_equal(got, want), k


def test_softmax_rows(ane, oracle):
    rng = np.random.default_rng(5)
    for n in (1, 5, 4096, 151936):
        x = (rng.standard_normal((3, n)) * 3).astype(np.float32)
        t = dev(x)
        ane.softmax_rows(t)
        want = oracle.softmax_rows(x)
        assert np.array_equal(t.cpu().numpy().view(np.int32), want.view(np.int32)), n
