"""GPU rmsnorm_gated, l2_normalize (core/cpu_ops.cpp:33-39, :106-111) and the
norm-weight loads (core/safetensors.cpp:264-306) through the C ABI: bit-exact
against the oracle (which is bit-exact against the reference in fp32)."""
import numpy as np
import pytest

from test_gpu_layer_ops import rand, to_dev, to_host

pytestmark = pytest.mark.gpu

DIMS = [128, 64, 100, 4096, 8192]


def _torch():
    import torch
    return torch


def bits(a):
    return a.view(np.uint32) if a.dtype == np.float32 else a.view(np.uint16)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("dim", DIMS)
def test_rmsnorm_gated(ane, oracle, dt, dim):
    rng = np.random.default_rng(dim * 3 + len(dt))
    rows = 37
    x = rand(rng, (rows, dim), dt, scale=2.0, outliers=0.01)
    z = rand(rng, (rows, dim), dt, scale=4.0, outliers=0.01)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    want = oracle.rmsnorm_gated(x, z, w)
    torch = _torch()
    got = ane.rmsnorm_gated(to_dev(x, dt), to_dev(z, dt), torch.from_numpy(w).cuda())
    assert np.array_equal(bits(to_host(got, dt)), bits(want))


def test_rmsnorm_gated_strided_in_place(ane, oracle):
    """Heads of a wider buffer, output over the input (per-head call of
    models/llm/qwen3_5.cpp:545-550)."""
    torch = _torch()
    rng = np.random.default_rng(4)
    buf = rng.standard_normal((16, 200)).astype(np.float32)
    z = rng.standard_normal((16, 128)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    want = oracle.rmsnorm_gated(np.ascontiguousarray(buf[:, :128]), z, w)
    d = torch.from_numpy(buf).cuda()
    ane.rmsnorm_gated(d[:, :128], torch.from_numpy(z).cuda(), torch.from_numpy(w).cuda(),
                      out=d[:, :128])
    got = d.cpu().numpy()
    assert np.array_equal(got[:, :128].view(np.uint32), want.view(np.uint32))
    assert np.array_equal(got[:, 128:], buf[:, 128:])


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("dim", DIMS)
@pytest.mark.parametrize("scale", [1.0, 1.0 / np.sqrt(128.0)], ids=["plain", "qscale"])
def test_l2_normalize(ane, oracle, dt, dim, scale):
    rng = np.random.default_rng(dim + 7)
    rows = 21
    x = rand(rng, (rows, dim), dt, scale=3.0)
    if dt == "f32":
        x[5] = 0.0  # a zero row stays zero (1 / sqrt(1e-12) * 0)
    want = oracle.l2_normalize(x, np.float32(scale))
    d = to_dev(x, dt)
    ane.l2_normalize(d, float(np.float32(scale)))
    assert np.array_equal(bits(to_host(d, dt)), bits(want))


@pytest.mark.parametrize("n,off", [(4096, 0), (1000003, 0), (77, 1)])
def test_bf16_weight_load(ane, oracle, n, off):
    torch = _torch()
    rng = np.random.default_rng(n)
    b = rng.integers(0, 1 << 16, n + off, dtype=np.uint64).astype(np.uint16)
    b[off:off + 5] = [0x7F80, 0xFF80, 0x7FC1, 0x8000, 0x3F80]
    d = torch.from_numpy(b.view(np.int16)).cuda()[off:]
    for add_one in (False, True):
        want = oracle.bf16_to_f32_weights(b[off:], add_one)
        got = ane.bf16_to_f32(d, add_one=add_one).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), add_one
