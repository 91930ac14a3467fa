"""GPU kernels of the next rows against the reference-generated fixtures in
tests/golden/ (decode attention, the hybrid row ops, the ANE-boundary
conversions, the norm-weight loads): the reference's own outputs, checked on
the GPU box where the reference tree is absent."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _torch():
    import torch
    return torch


def test_attention_golden(ane):
    """fp32 kernel within 1e-6 x max|v| of the reference's gqa_attention."""
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "gqa_attention.npz"))
    i = 0
    while f"q{i}" in g:
        q, k, v = (torch.from_numpy(g[f"{n}{i}"].astype(np.float32)).cuda()[None] for n in "qkv")
        start, ln, cap = (int(t) for t in g[f"ring{i}"])
        st = torch.tensor([start], dtype=torch.int32).cuda()
        n = torch.tensor([ln], dtype=torch.int32).cuda()
        got = ane.decode_attention(q, k, v, st, n).cpu().numpy()[0]
        assert np.abs(got - g[f"out{i}"]).max() <= 1e-6 * float(v.abs().max()), i
        i += 1
    assert i == 5


def test_hybrid_rows_golden(ane):
    """rmsnorm_gated and l2_normalize bit-exact with the reference (fp32)."""
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "hybrid_rows.npz"))
    x, z, w = (torch.from_numpy(g[n]).cuda() for n in ("x", "z", "w"))
    got = ane.rmsnorm_gated(x, z, w).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), g["gated"].view(np.uint32))
    y = x.clone()
    ane.l2_normalize(y)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), g["l2"].view(np.uint32))


def test_ane_convert_golden(ane):
    """Truncating pack and exact unpack bit-exact with the reference's
    f32_to_f16 / f16_to_f32 (spatial 1: one element per channel)."""
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "ane_convert.npz"))
    f32 = torch.from_numpy(g["f32"]).cuda().view(1, -1)
    s = ane.ane_pack(f32, round_mode=ane.ROUND_TRUNCATE, spatial=1)
    assert np.array_equal(s.cpu().numpy().view(np.uint16).ravel(), g["trunc"])
    h = torch.from_numpy(np.arange(65536, dtype=np.uint16).view(np.int16)).cuda().view(1, -1, 1)
    w = ane.ane_unpack(h, 1, spatial=1).cpu().numpy().ravel()
    assert np.array_equal(w.view(np.uint32), g["widen"].view(np.uint32))


def test_norm_weight_golden(ane):
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "norm_weight.npz"))
    b = torch.from_numpy(g["bf16"].view(np.int16)).cuda()
    for key, add in (("plain", False), ("norm", True)):
        got = ane.bf16_to_f32(b, add_one=add).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), g[key].view(np.uint32)), key
