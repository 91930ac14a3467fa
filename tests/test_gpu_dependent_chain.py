"""Back-to-back dependent launches.

Every kernel of the library is launched with programmatic stream
serialisation, so the next kernel on a stream may be dispatched while the
previous one is still running; each kernel waits (griddepcontrol.wait)
before its first global-memory access.  These tests run a decode-step
chain in which each kernel reads what the one before it wrote -- gather ->
residual + RMSNorm (reads the gathered rows) -> QK-norm + RoPE in place on
the normalised rows -> SiLU-gate of halves of those rows -- with no host
synchronisation in between, eagerly and replayed from a captured CUDA
graph, and check every intermediate bit for bit against the oracle chain
(fp32).  A torch copy kernel at the head of the graph also checks the wait
through a kernel launched without the attribute.  A second test runs the
decode step's KV write (QK-norm + RoPE writing q in place and k / v into
the ring) followed at once by decode attention over that ring, against the
same two calls with a device synchronisation between them."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROWS, HIDDEN, VOCAB = 8, 1024, 5000
NQ, NKV, HD = 4, 2, 128  # (4 + 2 + 2) x 128 = HIDDEN: the q/k/v layout over the normed rows


def _inputs(torch, seed):
    rng = np.random.default_rng(seed)
    table = (rng.standard_normal((VOCAB, HIDDEN)) * 0.5).astype(np.float16)
    ids = rng.integers(0, VOCAB, ROWS).astype(np.int32)
    x = rng.standard_normal((ROWS, HIDDEN)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32)
    pos = rng.integers(0, 4096, ROWS).astype(np.int32)
    return table, ids, x, w, pos


def _oracle_chain(oracle, table, ids, x, w, pos):
    xe, bad = oracle.embedding_gather(table, ids, out_dtype=0)
    assert bad == 0
    x_after, y = oracle.residual_rmsnorm(x, xe, w)
    y = oracle.qk_norm_rope(y, NQ, NKV, HD, w[:HD], w[HD:2 * HD], pos, 1e6)
    h = oracle.silu_mul(np.ascontiguousarray(y[:, :HIDDEN // 2]),
                        np.ascontiguousarray(y[:, HIDDEN // 2:]))
    return xe, x_after, y, h


class _Chain:
    def __init__(self, torch, ane, table, ids, x, w, pos):
        self.torch, self.ane = torch, ane
        self.table = torch.from_numpy(table).cuda()
        self.ids = torch.from_numpy(ids).cuda()
        self.x0 = torch.from_numpy(x).cuda()
        self.x = self.x0.clone()
        self.w = torch.from_numpy(w).cuda()
        self.qw = self.w[:HD].clone()
        self.kw = self.w[HD:2 * HD].clone()
        self.pos = torch.from_numpy(pos).cuda()
        self.xe = torch.empty(ROWS, HIDDEN, device="cuda")
        self.y = torch.empty(ROWS, HIDDEN, device="cuda")
        self.h = torch.empty(ROWS, HIDDEN // 2, device="cuda")

    def run(self):
        ane, half = self.ane, HIDDEN // 2
        self.x.copy_(self.x0)  # a torch kernel, launched without the attribute
        ane.embedding_gather(self.table, self.ids, out_dtype=self.torch.float32, out=self.xe)
        ane.residual_rmsnorm(self.x, self.xe, self.w, out=self.y)
        ane.qk_norm_rope(self.y, self.qw, self.kw, self.pos, NQ, NKV, HD)
        ane.silu_mul(self.y[:, :half], self.y[:, half:], out=self.h)

    def results(self):
        return [t.cpu().numpy() for t in (self.xe, self.x, self.y, self.h)]


def _same(got, want):
    for name, g, e in zip(("gather", "residual", "qk", "silu"), got, want):
        assert np.array_equal(g.view(np.uint32), e.view(np.uint32)), name


def test_dependent_chain_eager(ane, oracle):
    import torch
    table, ids, x, w, pos = _inputs(torch, 41)
    want = _oracle_chain(oracle, table, ids, x, w, pos)
    ch = _Chain(torch, ane, table, ids, x, w, pos)
    for _ in range(3):  # repeated without synchronising in between
        ch.run()
    torch.cuda.synchronize()
    _same(ch.results(), want)


def test_dependent_chain_graph_replay(ane, oracle):
    import torch
    table, ids, x, w, pos = _inputs(torch, 42)
    want = _oracle_chain(oracle, table, ids, x, w, pos)
    ch = _Chain(torch, ane, table, ids, x, w, pos)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ch.run()  # warm-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ch.run()
    for _ in range(5):
        ch.y.zero_()
        ch.h.zero_()
        g.replay()
    torch.cuda.synchronize()
    _same(ch.results(), want)
    del g


def _decode_step_inputs(torch, seed, B=16, nq=32, nkv=8, hd=128, cap=1024):
    g = torch.Generator(device="cpu").manual_seed(seed)
    qkv = torch.randn(B, (nq + 2 * nkv) * hd, generator=g).half().cuda()
    kc = torch.randn(B, cap, nkv, hd, generator=g).half().cuda()
    vc = torch.randn(B, cap, nkv, hd, generator=g).half().cuda()
    start = torch.randint(0, cap, (B,), generator=g, dtype=torch.int32)
    ln = torch.randint(1, cap, (B,), generator=g, dtype=torch.int32)
    slots = ((start + ln) % cap).to(torch.int32)  # the new token's ring slot
    w = (1 + 0.1 * torch.randn(2, hd, generator=g)).float().cuda()
    pos = ln.clone()
    return dict(qkv=qkv, kc=kc, vc=vc, start=start.cuda(), ln=(ln + 1).cuda(), slots=slots.cuda(),
                qw=w[0].clone(), kw=w[1].clone(), pos=pos.cuda(), nq=nq, nkv=nkv, hd=hd)


def _decode_step(torch, ane, t, sync_between):
    B = t["qkv"].shape[0]
    ane.qk_norm_rope_kv(t["qkv"], t["qw"], t["kw"], t["pos"], t["nq"], t["nkv"], t["hd"],
                        t["kc"], t["vc"], t["slots"])
    if sync_between:
        torch.cuda.synchronize()
    q = t["qkv"][:, :t["nq"] * t["hd"]].view(B, t["nq"], t["hd"])
    return ane.decode_attention(q, t["kc"], t["vc"], t["start"], t["ln"])


def test_decode_step_kv_write_then_attention(ane):
    """The decode step's QK-norm + RoPE writes q in place and the new k / v
    into the ring; attention, launched right after, reads both (q through
    the read-only path, the ring through asynchronous copies).  Same bits as
    with a device synchronisation between the two."""
    import torch
    base = _decode_step_inputs(torch, 43)
    want_t = {k: (v.clone() if hasattr(v, "clone") else v) for k, v in base.items()}
    want = _decode_step(torch, ane, want_t, sync_between=True)
    torch.cuda.synchronize()
    for _ in range(3):
        t = {k: (v.clone() if hasattr(v, "clone") else v) for k, v in base.items()}
        got = _decode_step(torch, ane, t, sync_between=False)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
        assert torch.equal(t["kc"].view(torch.int16), want_t["kc"].view(torch.int16))
        assert torch.equal(t["vc"].view(torch.int16), want_t["vc"].view(torch.int16))

    # the same step replayed from a captured graph, inputs restored inside it
    t = {k: (v.clone() if hasattr(v, "clone") else v) for k, v in base.items()}
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        _decode_step(torch, ane, t, sync_between=False)  # warm-up (workspace, instances)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for key in ("qkv", "kc", "vc"):
            t[key].copy_(base[key])
        out = _decode_step(torch, ane, t, sync_between=False)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    del g


def test_prefill_chain_dependent_fp16_bulk_sizes(ane):
    """The prefill chain at sizes that take the register RMSNorm, the
    row-per-warp QK-norm + RoPE and the bulk-copy SiLU-gate -- the three
    kernels that prefetch their first inputs into L2 before waiting for the
    previous kernel -- with each kernel reading what the one before it is
    still writing: x += d and y = rmsnorm(x); QK-norm + RoPE in place on y;
    h = silu(y) * x over the whole rows (contiguous, so SiLU takes the bulk
    path).  Three chains back to back with no synchronisation, and the chain
    replayed from a captured graph, give the same bits as the same calls
    with a device synchronisation after each."""
    import torch
    R, H, nq, nkv, hd = 2048, 4096, 24, 8, 128  # (24 + 8) x 128 = H: q and k heads over y
    g = torch.Generator(device="cpu").manual_seed(44)
    x0 = torch.randn(R, H, generator=g).half().cuda()
    d = torch.randn(R, H, generator=g).half().cuda()
    w = (1 + 0.1 * torch.randn(H, generator=g)).float().cuda()
    qw = (1 + 0.1 * torch.randn(hd, generator=g)).float().cuda()
    kw = (1 + 0.1 * torch.randn(hd, generator=g)).float().cuda()
    pos = (torch.arange(R, dtype=torch.int32) % 512).cuda()

    def chain(x, y, h, sync):
        ane.residual_rmsnorm(x, d, w, out=y)
        if sync:
            torch.cuda.synchronize()
        ane.qk_norm_rope(y, qw, kw, pos, nq, nkv, hd)
        if sync:
            torch.cuda.synchronize()
        ane.silu_mul(y, x, out=h)
        if sync:
            torch.cuda.synchronize()

    xs, ys, hs = x0.clone(), torch.empty_like(x0), torch.empty_like(x0)
    want = []
    for _ in range(3):
        chain(xs, ys, hs, sync=True)
        want.append((xs.clone(), ys.clone(), hs.clone()))
    x, y, h = x0.clone(), torch.empty_like(x0), torch.empty_like(x0)
    got = []
    for _ in range(3):  # the next chain's RMSNorm reads the x this one wrote
        chain(x, y, h, sync=False)
        got.append((x.clone(), y.clone(), h.clone()))  # torch copies, launched without the attribute
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(got, want)):
        for name, t, e in zip(("x", "y", "h"), a, b):
            assert torch.equal(t.view(torch.int16), e.view(torch.int16)), (i, name)

    # replayed from a graph, the inputs restored inside it
    s = torch.cuda.Stream()
    x, y, h = x0.clone(), torch.empty_like(x0), torch.empty_like(x0)
    with torch.cuda.stream(s):
        chain(x, y, h, sync=False)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=s):
        x.copy_(x0)
        chain(x, y, h, sync=False)
    for _ in range(3):
        y.zero_()
        h.zero_()
        gr.replay()
    torch.cuda.synchronize()
    for name, t, e in zip(("x", "y", "h"), (x, y, h), want[0]):
        assert torch.equal(t.view(torch.int16), e.view(torch.int16)), ("graph", name)
    del gr
