"""GPU parity: BF16->FP16 conversion and embedding gather, through the C ABI,
bit-exact against the oracle and the reference-generated golden table."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _torch():
    import torch
    return torch


def test_convert_exhaustive_golden(ane):
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "bf16_to_f16.npz"))
    inp = torch.from_numpy(g["bf16"].view(np.int16)).cuda()
    out = ane.bf16_to_f16(inp)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), g["f16"])


@pytest.mark.parametrize("n,offset", [(1, 0), (7, 0), (8, 0), (1000003, 0), (4096, 1),
                                      (65541, 3), (1 << 20, 0),
                                      # long enough for the bulk-copy ring, ending mid-tile;
                                      # 16-byte aligned and unaligned starts
                                      (10000005, 0), (10000005, 8), (10000005, 3)])
def test_convert_ragged_and_unaligned(ane, oracle, n, offset):
    torch = _torch()
    rng = np.random.default_rng(n + offset)
    host = rng.integers(0, 65536, size=n + offset, dtype=np.uint16)
    dev = torch.from_numpy(host.view(np.int16)).cuda()
    src = dev[offset:]
    out_buf = torch.empty(n + offset, dtype=torch.int16, device="cuda")
    out = out_buf[offset:]
    ane.bf16_to_f16(src, out=out)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), oracle.bf16_to_f16(host[offset:]))


def test_convert_full_size_lut_property(ane):
    """1 G elements: every output equals the golden table at its input."""
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "bf16_to_f16.npz"))
    lut = torch.from_numpy(g["f16"].astype(np.int64)).cuda()
    n = 1 << 30
    gen = torch.Generator(device="cuda").manual_seed(5)
    inp = torch.randint(-32768, 32768, (n,), dtype=torch.int32, device="cuda", generator=gen)
    inp = inp.to(torch.int16)
    out = ane.bf16_to_f16(inp)
    want = lut[inp.to(torch.int64) & 0xFFFF].to(torch.int32)
    got = out.to(torch.int32) & 0xFFFF
    assert torch.equal(got, want)


@pytest.mark.parametrize("tdt,hidden", [("f16", 1024), ("f32", 1024), ("bf16", 4096),
                                        ("f16", 100), ("f16", 4)])
def test_gather_vs_oracle(ane, oracle, tdt, hidden):
    torch = _torch()
    rng = np.random.default_rng(hidden)
    vocab = 3000
    npdt = {"f16": np.float16, "f32": np.float32, "bf16": np.uint16}[tdt]
    if tdt == "bf16":
        table = rng.integers(0, 65536, size=(vocab, hidden), dtype=np.uint16)
        tt = torch.from_numpy(table.view(np.int16)).cuda().view(torch.bfloat16)
    else:
        table = rng.standard_normal((vocab, hidden)).astype(npdt)
        tt = torch.from_numpy(table).cuda()
    ids = rng.integers(0, vocab, size=257).astype(np.int32)
    got = ane.embedding_gather(tt, torch.from_numpy(ids).cuda())
    want, bad = oracle.embedding_gather(table, ids)
    assert bad == 0
    g = got.cpu()
    g = g.view(torch.int16).numpy().view(np.uint16) if tdt == "bf16" else g.numpy()
    assert np.array_equal(g.view(np.uint8), want.view(np.uint8))
    if tdt != "f32":
        got32 = ane.embedding_gather(tt, torch.from_numpy(ids).cuda(), out_dtype=torch.float32)
        want32, _ = oracle.embedding_gather(table, ids, out_dtype=0)
        # compare bit patterns: random BF16 inputs include NaNs
        assert np.array_equal(got32.cpu().numpy().view(np.uint32), want32.view(np.uint32))


def test_gather_bad_ids_zero_row_and_flag(ane):
    torch = _torch()
    ane.read_status_flags(clear=True)
    table = torch.randn(50, 64, device="cuda", dtype=torch.float16)
    ids = torch.tensor([3, -1, 50, 49], dtype=torch.int32, device="cuda")
    out = ane.embedding_gather(table, ids)
    assert ane.read_status_flags(clear=True) & ane.FLAG_BAD_TOKEN_ID
    assert torch.equal(out[0], table[3]) and torch.equal(out[3], table[49])
    assert not out[1].any() and not out[2].any()
    ane.embedding_gather(table, ids[:1])
    assert ane.read_status_flags(clear=True) == 0


def test_decode_gather_qwen3_06b(ane, oracle):
    """Config 1: one token from an fp16 151936 x 1024 table into an fp32 row."""
    torch = _torch()
    gen = torch.Generator(device="cuda").manual_seed(1)
    table = (torch.randn(151936, 1024, device="cuda", generator=gen) * 0.02).half()
    tok = 151935
    out = ane.embedding_gather(table, torch.tensor([tok], dtype=torch.int32, device="cuda"),
                               out_dtype=torch.float32)
    assert torch.equal(out[0], table[tok].float())
