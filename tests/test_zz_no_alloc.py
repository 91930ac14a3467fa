"""The allocation-free decode attention (ane_cuda_decode_attention_static):
same results as ane_cuda_decode_attention, no device memory allocated per
call, problems beyond its fixed scratch rejected.  Collected last so it also
runs after every other GPU test in the same process."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-6  # x max|v|; the two entry points run the same kernel, so 0 in practice


def _case(torch, B, H, hk, hd, cap, starts, lens, dt, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, H, hd, generator=g).to(dt).cuda()
    k = torch.randn(B, cap, hk, hd, generator=g).to(dt).cuda()
    v = torch.randn(B, cap, hk, hd, generator=g).to(dt).cuda()
    st = torch.tensor(starts, dtype=torch.int32).cuda()
    ln = torch.tensor(lens, dtype=torch.int32).cuda()
    return q, k, v, st, ln


@pytest.mark.parametrize("dt_name", ["float32", "float16"])
def test_static_matches_regular_two_calls(ane, dt_name):
    import torch
    dt = getattr(torch, dt_name)
    q, k, v, st, ln = _case(torch, 2, 32, 8, 128, 2048, [100, 0], [2048, 777], dt, 5)
    want = ane.decode_attention(q, k, v, st, ln).float()
    vmax = v.float().abs().max().item()
    for _ in range(2):  # the second call finds the first call's partials in the array
        got = ane.decode_attention_static(q, k, v, st, ln).float()
        torch.cuda.synchronize()
        assert (got - want).abs().max().item() <= TOL * vmax


def test_static_allocates_nothing(ane):
    import torch
    q, k, v, st, ln = _case(torch, 1, 16, 8, 128, 4096, [9], [4096], torch.float32, 6)
    out = torch.empty_like(q)
    ane.decode_attention_static(q, k, v, st, ln, out=out)  # first use loads the image
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        ane.decode_attention_static(q, k, v, st, ln, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_static_rejects_beyond_capacity(ane):
    import torch
    cap_bytes = ane.lib().ane_cuda_decode_attention_static_capacity()
    assert cap_bytes > 0
    B, H, hk, hd = 64, 32, 8, 128
    max_len = 8192
    assert ane.decode_attention_workspace_size(B, H, hk, hd, max_len) > cap_bytes
    q = torch.zeros(B, H, hd, device="cuda")
    k = torch.zeros(B, 64, hk, hd, device="cuda")
    st = torch.zeros(B, dtype=torch.int32, device="cuda")
    with pytest.raises(ane.AneCudaError) as e:
        ane.decode_attention_static(q, k, k, st, st, max_len=max_len)
    assert e.value.status == ane.ERR_INVALID_ARG
