"""GPU fp32 <-> fp16 packing at the ANE boundary (core/ane_runtime.cpp:611-653)
through the C ABI: bit-exact against the oracle in both rounding modes, with
untouched spatial slots preserved."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


def values(rng, shape):
    x = rng.standard_normal(shape).astype(np.float32) * np.float32(300)
    flat = x.reshape(-1)
    n = flat.size
    k = max(1, n // 50)
    idx = rng.choice(n, size=min(n, 8 * k), replace=False)
    specials = np.array([np.inf, -np.inf, np.nan, -np.nan, 0.0, -0.0, 65504.0, 65519.99, 65520.0,
                         1e6, -1e6, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8, 1e-10, -3e-7,
                         65536.0, -65536.0, 65535.996, -65535.996, 3.4e38], np.float32)
    flat[idx[:k]] = rng.choice(specials, k)
    flat[idx[k:2 * k]] = rng.standard_normal(k).astype(np.float32) * np.float32(1e-5)  # subnormal range
    flat[idx[2 * k:3 * k]] = (rng.integers(0, 1 << 32, k, dtype=np.uint64).astype(np.uint32)).view(np.float32)
    return x


CASES = [  # tokens, channels, in_stride extra, spatial
    (1, 1024, 0, 32),      # Qwen3-0.6B decode token
    (32, 4096, 0, 32),     # one full surface
    (45, 1000, 0, 32),     # ragged tokens and channels
    (100, 130, 0, 32),     # partial channel chunk
    (64, 256, 3, 32),      # strided, unaligned rows -> scalar loads
    (40, 96, 0, 16),       # another spatial size -> generic path
]


@pytest.mark.parametrize("round_mode", [0, 1], ids=["nearest", "truncate"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"t{c[0]}c{c[1]}s{c[2]}sp{c[3]}")
def test_pack_matches_oracle(ane, oracle, round_mode, case):
    torch = _torch()
    t, c, extra, sp = case
    rng = np.random.default_rng(t * 7919 + c)
    x = values(rng, (t, c + extra))
    nsurf = (t + sp - 1) // sp
    base = rng.integers(0, 1 << 16, (nsurf, c, sp), dtype=np.uint64).astype(np.uint16)
    want = oracle.ane_pack(np.ascontiguousarray(x[:, :c]), round_mode=round_mode, spatial=sp,
                           surface=base)
    xd = torch.from_numpy(x).cuda()[:, :c]
    sd = torch.from_numpy(base.view(np.int16)).cuda()
    ane.ane_pack(xd, round_mode=round_mode, spatial=sp, surface=sd)
    got = sd.cpu().numpy().view(np.uint16)
    assert np.array_equal(got, want), f"{int((got != want).sum())} elements differ"


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"t{c[0]}c{c[1]}s{c[2]}sp{c[3]}")
def test_unpack_matches_oracle(ane, oracle, case):
    torch = _torch()
    t, c, extra, sp = case
    rng = np.random.default_rng(t + c)
    nsurf = (t + sp - 1) // sp
    surf = rng.integers(0, 1 << 16, (nsurf, c, sp), dtype=np.uint64).astype(np.uint16)
    want = oracle.ane_unpack(surf, t, spatial=sp)
    out = torch.full((t, c + extra), 7.0, device="cuda")
    ane.ane_unpack(torch.from_numpy(surf.view(np.int16)).cuda(), t, spatial=sp, out=out[:, :c])
    got = out.cpu().numpy()
    assert np.array_equal(got[:, :c].view(np.uint32), want.view(np.uint32))
    assert np.all(got[:, c:] == 7.0)


def test_pack_unaligned_surface(ane, oracle):
    """A surface that is not 16-byte aligned takes the generic path."""
    torch = _torch()
    rng = np.random.default_rng(3)
    x = values(rng, (33, 64))
    want = oracle.ane_pack(x)
    buf = torch.zeros(2 * 64 * 32 + 1, dtype=torch.int16, device="cuda")
    sd = buf[1:].view(2, 64, 32)
    ane.ane_pack(torch.from_numpy(x).cuda(), surface=sd)
    assert np.array_equal(sd.cpu().numpy().view(np.uint16), want)


def test_pack_unpack_round_trip_large(ane):
    """Qwen3-8B hidden size over 4096 tokens: unpack(pack(x)) is x rounded to
    fp16 (checked against torch's own conversion for finite values)."""
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(4096, 4096, device="cuda", generator=g) * 10
    s = ane.ane_pack(x)
    y = ane.ane_unpack(s, 4096)
    assert torch.equal(y, x.half().float())
    assert torch.equal(s.view(torch.float16)[0, :, 5].float(), x[5].half().float())


def test_pack_rejects_bad_args(ane):
    torch = _torch()
    x = torch.zeros(4, 8, device="cuda")
    with pytest.raises(ane.AneCudaError):
        ane.ane_pack(x, round_mode=2)
    st = ane.lib().ane_cuda_ane_pack(0, None, None, 8, 4, 8, 0, None)
    assert st == ane.ERR_INVALID_ARG
