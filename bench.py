"""Benchmark of the ANE-LM layer-op hot path on B200.

Headline (BASELINE metric "fused-layer-op HBM GB/s (% of B200 peak) and
rows/s"): the Qwen3-8B batched-prefill layer-op chain -- residual add +
RMSNorm, per-head QK-norm + RoPE, SiLU-gate -- over 64 x 512 = 32768 rows
per GPU (weak scaling: every rank runs the full config on its own rows, no
collective on the data path).  A step is one pass of the three kernels over
all rows.  Synthetic fp16 ~N(0,1) activations with 0.1% of entries x50,
positions row mod 512.  Every kernel's inputs exceed the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line.  --impl reference times the reference's own CPU
code for the same chain (oracle/_ref, the reference sources compiled here;
the C restatement when that build is absent) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "ane-lm_b200")

# Qwen3-8B batched prefill
ROWS, HIDDEN, NQ, NKV, HD, INTER = 32768, 4096, 32, 8, 128, 12288
SEQ = 512
THETA, EPS = 1e6, 1e-6
# algorithmic bytes per row (fp16): resid+norm reads x, d and writes x, y;
# QK-norm+RoPE reads and writes the q and k heads; SiLU reads gate, up and
# writes h.
B_NORM = 4 * HIDDEN * 2
B_QK = (NQ + NKV) * HD * 2 * 2
B_SILU = 3 * INTER * 2
B_ROW = B_NORM + B_QK + B_SILU            # 126,976
FALLBACK_HBM_GBS = 6650.0


def measured_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def rank_rows(rank, rows_per_rank=None):
    """Weak scaling: rank r owns global rows [r * R, (r + 1) * R) of the
    batched-prefill chain (R = ROWS).  Rows are independent, so a rank's
    inputs come from the seed and its row offset and nothing crosses ranks
    on the data path."""
    r = ROWS if rows_per_rank is None else rows_per_rank
    return rank * r, r


def chain_seed(row0):
    """Seed of a rank's synthetic inputs: the base seed plus its row offset."""
    return 1234 + row0


def aggregate_gbs(world, rows_per_rank, ms):
    """Whole-job GB/s of the chain: every rank's rows over the slowest rank's time."""
    return world * rows_per_rank * B_ROW / (ms * 1e-3) / 1e9


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in (self.out or "").splitlines():
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() in ("active", "1"):
                    reasons.add(nm)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        sms.sort()
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def _setup_gpu(world):
    import torch
    import torch.distributed as dist
    rank, local, _ = env_rank()
    torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    sys.path.insert(0, PKG)
    import ane_lm_cuda
    ane_lm_cuda.lib()  # fails loudly when the library is missing
    return torch, ane_lm_cuda, rank, local


def make_chain_inputs(torch, rows, hidden, nq, nkv, hd, inter, seq, seed):
    """fp16 ~N(0,1) with 0.1% of entries x50; positions row mod seq."""
    g = torch.Generator(device="cuda").manual_seed(seed)

    def act(*shape):
        a = torch.randn(*shape, device="cuda", generator=g, dtype=torch.float32)
        m = torch.rand(*shape, device="cuda", generator=g) < 1e-3
        a[m] *= 50.0
        return a.half()

    b = {
        "x": act(rows, hidden), "d": act(rows, hidden),
        "y": torch.empty(rows, hidden, device="cuda", dtype=torch.float16),
        "w": (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).float(),
        "qkv": act(rows, (nq + 2 * nkv) * hd),
        "qw": (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).float(),
        "kw": (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).float(),
        "pos": (torch.arange(rows, device="cuda", dtype=torch.int32) % seq),
        "gate": act(rows, inter), "up": act(rows, inter),
        "h": torch.empty(rows, inter, device="cuda", dtype=torch.float16),
    }
    return b


class Chain:
    """The three layer-op launches of one step, through the C ABI."""

    def __init__(self, ane, b, rows, hidden, nq, nkv, hd, inter, stream_ptr):
        import ctypes as C
        self.L = ane.lib()
        P = lambda t, off=0: C.c_void_p(t.data_ptr() + off)  # noqa: E731
        width = (nq + 2 * nkv) * hd
        s = C.c_void_p(stream_ptr)
        self.norm = (1, P(b["x"]), hidden, P(b["d"]), hidden, P(b["y"]), hidden, P(b["w"]),
                     rows, hidden, EPS, s)
        self.qk = (1, P(b["qkv"]), P(b["qkv"], nq * hd * 2), width, width, hd, hd, nq, nkv, hd, hd,
                   P(b["qw"]), P(b["kw"]), P(b["pos"]), rows, THETA, EPS, s)
        self.silu = (1, P(b["h"]), inter, P(b["gate"]), inter, P(b["up"]), inter, rows, inter, s)

    def launch(self, ev=None):
        L = self.L
        if ev is not None:
            ev[0].record()
        st = L.ane_cuda_residual_rmsnorm(*self.norm)
        if ev is not None:
            ev[1].record()
        st |= L.ane_cuda_qk_norm_rope(*self.qk)
        if ev is not None:
            ev[2].record()
        st |= L.ane_cuda_silu_mul(*self.silu)
        if ev is not None:
            ev[3].record()
        if st:
            raise RuntimeError("kernel launch failed: " + L.ane_cuda_last_error().decode())


def time_device_chain(torch, dist, world, chain, steps, warmup, gpu_index):
    for _ in range(warmup):
        chain.launch()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpu_index) as clk:
        start.record()
        for i in range(steps):
            chain.launch(evs[i])
        end.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    total_ms = start.elapsed_time(end)
    per = [0.0, 0.0, 0.0]
    for e in evs:
        for k in range(3):
            per[k] += e[k].elapsed_time(e[k + 1])
    per = [p / steps for p in per]
    return total_ms, per, clk.summary()


def max_over_ranks(torch, dist, world, v):
    """The slowest rank's value: a one-element MAX all-reduce (the timing
    collective, never on the data path); on the CPU backend (gloo) too."""
    if world == 1:
        return v
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_e2e_chain(torch, ane, rows, steps, chunks=8):
    """The same chain through the public C ABI with HOST buffers: every step
    copies its inputs (x, d, qkv, gate, up) from pinned memory to the device,
    runs the three kernels and copies the outputs (x, y, qkv, h) back, in
    `chunks` row blocks over two streams so copies overlap the kernels."""
    import ctypes as C
    L = ane.lib()
    width = (NQ + 2 * NKV) * HD
    pin = dict(pin_memory=True)
    g = torch.Generator().manual_seed(7)
    hx = (torch.randn(rows, HIDDEN, generator=g)).half().pin_memory()
    hd_ = (torch.randn(rows, HIDDEN, generator=g)).half().pin_memory()
    hq = (torch.randn(rows, width, generator=g)).half().pin_memory()
    hg = (torch.randn(rows, INTER, generator=g)).half().pin_memory()
    hu = (torch.randn(rows, INTER, generator=g)).half().pin_memory()
    oy = torch.empty(rows, HIDDEN, dtype=torch.float16, **pin)
    oh = torch.empty(rows, INTER, dtype=torch.float16, **pin)
    w = torch.ones(HIDDEN, device="cuda")
    qw = torch.ones(HD, device="cuda")
    pos = (torch.arange(rows, device="cuda", dtype=torch.int32) % SEQ)
    cr = rows // chunks
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    dev = [{k: torch.empty(cr, n, device="cuda", dtype=torch.float16)
            for k, n in (("x", HIDDEN), ("d", HIDDEN), ("y", HIDDEN), ("q", width),
                         ("g", INTER), ("u", INTER), ("h", INTER))} for _ in streams]
    P = lambda t, off=0: C.c_void_p(t.data_ptr() + off)  # noqa: E731

    def step():
        for c in range(chunks):
            s = streams[c % 2]
            b = dev[c % 2]
            r0, r1 = c * cr, (c + 1) * cr
            with torch.cuda.stream(s):
                b["x"].copy_(hx[r0:r1], non_blocking=True)
                b["d"].copy_(hd_[r0:r1], non_blocking=True)
                b["q"].copy_(hq[r0:r1], non_blocking=True)
                b["g"].copy_(hg[r0:r1], non_blocking=True)
                b["u"].copy_(hu[r0:r1], non_blocking=True)
                sp = C.c_void_p(s.cuda_stream)
                st = L.ane_cuda_residual_rmsnorm(1, P(b["x"]), HIDDEN, P(b["d"]), HIDDEN, P(b["y"]),
                                                 HIDDEN, P(w), cr, HIDDEN, EPS, sp)
                st |= L.ane_cuda_qk_norm_rope(1, P(b["q"]), P(b["q"], NQ * HD * 2), width, width,
                                              HD, HD, NQ, NKV, HD, HD, P(qw), P(qw), P(pos, r0 * 4),
                                              cr, THETA, EPS, sp)
                st |= L.ane_cuda_silu_mul(1, P(b["h"]), INTER, P(b["g"]), INTER, P(b["u"]), INTER,
                                          cr, INTER, sp)
                if st:
                    raise RuntimeError(L.ane_cuda_last_error().decode())
                hx[r0:r1].copy_(b["x"], non_blocking=True)
                oy[r0:r1].copy_(b["y"], non_blocking=True)
                hq[r0:r1].copy_(b["q"], non_blocking=True)
                oh[r0:r1].copy_(b["h"], non_blocking=True)

    cur = torch.cuda.current_stream()
    step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(cur)
    for s in streams:
        s.wait_stream(cur)
    for _ in range(steps):
        step()
    for s in streams:
        cur.wait_stream(s)
    end.record(cur)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    h2d = rows * (2 * HIDDEN + width + 2 * INTER) * 2
    d2h = rows * (2 * HIDDEN + width + INTER) * 2
    return ms, h2d, d2h, 3 * chunks * steps


def time_extras(torch, ane, reps=20):
    """Secondary configs (per GPU): BF16->FP16 convert of a Qwen3-8B-shaped
    checkpoint (flat), the 256-row sampler, the Qwen3-1.7B prefill chain,
    the Qwen3-0.6B batch-1 decode chain latency, decode attention and the
    ANE-boundary packing."""
    import ctypes as C
    L = ane.lib()
    out = {}
    cur = torch.cuda.current_stream()
    sp = C.c_void_p(cur.cuda_stream)
    P = lambda t, off=0: C.c_void_p(t.data_ptr() + off)  # noqa: E731

    def timed(fn, n):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    # convert: embedding + 36 layers (q, k, v, o, gate, up, down) + lm_head
    params = 151936 * 4096 * 2 + 36 * (4096 * 4096 * 2 + 1024 * 4096 * 2 + 12288 * 4096 * 3)
    src = torch.randint(-32768, 32768, (params,), dtype=torch.int16, device="cuda")
    dst = torch.empty_like(src)
    ms = timed(lambda: L.ane_cuda_bf16_to_f16(P(dst), P(src), params, sp), reps)
    out["convert_qwen3_8b"] = {"params": params, "ms": round(ms, 4),
                               "gb_s": round(params * 4 / ms / 1e6, 1)}
    del src, dst

    # sampler: 256 x 151936
    rows, vocab = 256, 151936
    g = torch.Generator(device="cuda").manual_seed(3)
    logits = torch.randn(rows, vocab, device="cuda", generator=g) * 3
    hist = torch.randint(0, vocab, (rows, 1024), device="cuda", dtype=torch.int32, generator=g)
    hlen = torch.full((rows,), 1024, device="cuda", dtype=torch.int32)
    u = torch.rand(rows, device="cuda", generator=g)
    tok = torch.empty(rows, device="cuda", dtype=torch.int32)
    ms = timed(lambda: L.ane_cuda_sample_rows(P(logits), rows, vocab, vocab, P(hist), P(hlen), 1024,
                                              P(u), 0.6, 1.2, 256, 0.1, P(tok), sp), reps)
    by = rows * (vocab * 4 + 1024 * 4 + 4 + 4)
    out["sampler_256x151936"] = {"ms": round(ms, 4), "rows_per_s": round(rows / ms * 1e3, 1),
                                 "gb_s": round(by / ms / 1e6, 1)}
    del logits

    # Qwen3-1.7B prefill chain, T = 2048
    b = make_chain_inputs(torch, 2048, 2048, 16, 8, 128, 6144, 2048, 5)
    ch = Chain(ane, b, 2048, 2048, 16, 8, 128, 6144, cur.cuda_stream)
    ms = timed(ch.launch, reps * 5)
    out["prefill_qwen3_1p7b_t2048"] = {"ms": round(ms, 4),
                                       "gb_s": round(2048 * 65536 / ms / 1e6, 1)}
    del b, ch

    # Qwen3-0.6B decode, batch 1: gather (fp16 table -> fp32 row), resid+norm,
    # QK-norm+RoPE and SiLU-gate in fp32, replayed as one CUDA graph
    table = (torch.randn(151936, 1024, device="cuda", generator=g) * 0.02).half()
    tid = torch.randint(0, 151936, (1,), device="cuda", dtype=torch.int32, generator=g)
    xe = torch.empty(1, 1024, device="cuda")
    x = torch.randn(1, 1024, device="cuda", generator=g)
    y = torch.empty_like(x)
    w = torch.ones(1024, device="cuda")
    qkv = torch.randn(1, (16 + 16) * 128, device="cuda", generator=g)
    pos = torch.randint(0, 4096, (1,), device="cuda", dtype=torch.int32, generator=g)
    ga, up, h = (torch.randn(1, 3072, device="cuda", generator=g) for _ in range(3))
    gs = torch.cuda.Stream()

    def decode(stream):
        s = C.c_void_p(stream.cuda_stream)
        st = L.ane_cuda_embedding_gather(P(xe), 0, P(table), 1, P(tid), 1, 151936, 1024, s)
        st |= L.ane_cuda_residual_rmsnorm(0, P(x), 1024, P(xe), 1024, P(y), 1024, P(w), 1, 1024,
                                          EPS, s)
        st |= L.ane_cuda_qk_norm_rope(0, P(qkv), P(qkv, 16 * 128 * 4), 4096, 4096, 128, 128, 16, 8,
                                      128, 128, P(w), P(w), P(pos), 1, THETA, EPS, s)
        st |= L.ane_cuda_silu_mul(0, P(h), 3072, P(ga), 3072, P(up), 3072, 1, 3072, s)
        if st:
            raise RuntimeError(L.ane_cuda_last_error().decode())

    with torch.cuda.stream(gs):
        decode(gs)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        decode(gs)
    ms = timed(graph.replay, 200)
    del graph
    # the same step 16 times in one graph: the host's graph launches, which
    # the one-step replays above also measure, are amortised as they are in
    # a whole-model graph
    graph16 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph16, stream=gs):
        for _ in range(16):
            decode(gs)
    ms16 = timed(graph16.replay, 25) / 16
    del graph16
    out["decode_qwen3_0p6b_b1"] = {"us_per_token": round(ms * 1e3, 2),
                                   "us_per_step_in_16_step_graph": round(ms16 * 1e3, 2),
                                   "kernels": 4}

    # decode attention over the KV ring: Qwen3-0.6B batch 1 with the
    # reference's fp32 cache, and Qwen3-8B batch 64 with an fp16 cache; 4096
    # keys, ring start mid-cache (wrapped).  CUDA graph of back-to-back calls
    # over rotating cache copies (more than L2 in total).
    peak, _ = measured_peak()
    for name, (B, H, hk, dt) in {"attention_qwen3_0p6b_b1_l4096_f32": (1, 16, 8, torch.float32),
                                 "attention_qwen3_8b_b64_l4096_f16": (64, 32, 8, torch.float16)}.items():
        us, gbs = time_attention(torch, ane, B, H, hk, 128, 4096, dt)
        out[name] = {"us": round(us, 2), "gb_s": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4)}

    # fp32 <-> fp16 packing at the ANE boundary: 32,768 tokens x 4096
    # channels (1,024 surfaces of [4096][32]); 6 bytes per (token, channel)
    T, Cn = 32768, 4096
    x = torch.randn(T, Cn, device="cuda", generator=g)
    surf = torch.zeros((T // 32, Cn, 32), dtype=torch.int16, device="cuda")
    y = torch.empty_like(x)
    for name, fn in (("ane_pack_32k_x_4096", lambda: ane.ane_pack(x, surface=surf)),
                     ("ane_unpack_32k_x_4096", lambda: ane.ane_unpack(surf, T, out=y))):
        ms = timed(fn, reps)
        gbs = T * Cn * 6 / ms / 1e6
        out[name] = {"us": round(ms * 1e3, 2), "gb_s": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4)}
    del x, surf, y
    return out


def time_attention(torch, ane, B, H, hk, hd, ln, dt, start=1000):
    """(us per call, GB/s of K and V read) for ane.decode_attention."""
    es = torch.tensor([], dtype=dt).element_size()
    kv_bytes = 2 * B * ln * hk * hd * es
    ncopy = max(1, min(16, (512 << 20) // kv_bytes + 1))
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(B, H, hd, device="cuda", generator=g).to(dt)
    ks = [torch.randn(B, ln, hk, hd, device="cuda", generator=g).to(dt) for _ in range(ncopy)]
    vs = [torch.randn(B, ln, hk, hd, device="cuda", generator=g).to(dt) for _ in range(ncopy)]
    st = torch.full((B,), start, dtype=torch.int32, device="cuda")
    ln_t = torch.full((B,), ln, dtype=torch.int32, device="cuda")
    ws = torch.zeros(max(1, ane.decode_attention_workspace_size(B, H, hk, hd, ln)),
                     dtype=torch.uint8, device="cuda")
    out = torch.empty_like(q)
    s = torch.cuda.Stream()
    reps = ncopy * max(1, 32 // ncopy)
    with torch.cuda.stream(s):
        for i in range(3):
            ane.decode_attention(q, ks[i % ncopy], vs[i % ncopy], st, ln_t, max_len=ln, out=out,
                                 workspace=ws)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(reps):
                ane.decode_attention(q, ks[i % ncopy], vs[i % ncopy], st, ln_t, max_len=ln,
                                     out=out, workspace=ws)
        graph.replay()
        s.synchronize()
        ts = []
        for _ in range(10):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            graph.replay()
            b.record(s)
            b.synchronize()
            ts.append(a.elapsed_time(b) / reps)
    ts.sort()
    ms = ts[len(ts) // 2]
    del graph
    return ms * 1e3, kv_bytes / ms / 1e6


# ---------------------------------------------------------------------------
# CPU: the reference's own chain (oracle/_ref) or the C restatement
# ---------------------------------------------------------------------------
class CpuChain:
    """Runs the layer-op chain over row blocks of host buffers on N threads
    (ctypes releases the GIL, so the threads run in parallel)."""

    def __init__(self, rows):
        import numpy as np
        sys.path.insert(0, os.path.join(REPO, "tests"))
        from oracle_lib import Oracle, load_ref
        self.np = np
        self.ref = load_ref()
        self.kind = "reference" if self.ref is not None else "port"
        self.orc = None if self.ref is not None else Oracle().lib
        rng = np.random.default_rng(17)
        width = (NQ + 2 * NKV) * HD

        def act(*shape):
            a = rng.standard_normal(shape, dtype=np.float32)
            a[rng.random(shape) < 1e-3] *= 50.0
            return a.astype(np.float16)

        self.rows = rows
        self.x, self.d = act(rows, HIDDEN), act(rows, HIDDEN)
        self.y = np.empty_like(self.x)
        self.w = (1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32)
        self.qkv = act(rows, width)
        self.qw = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
        self.kw = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
        self.pos = (np.arange(rows) % SEQ).astype(np.int32)
        self.g, self.u = act(rows, INTER), act(rows, INTER)
        self.h = np.empty_like(self.g)

    def run_block(self, r0, r1):
        import ctypes as C
        p = lambda a, off=0: C.c_void_p(a.ctypes.data + off)  # noqa: E731
        if self.ref is not None:
            self.ref.ref_layer_chain_f16(p(self.x), p(self.d), p(self.y), p(self.w), p(self.qkv),
                                         p(self.qw), p(self.kw), p(self.pos), p(self.g), p(self.u),
                                         p(self.h), r0, r1, HIDDEN, NQ, NKV, HD, INTER, THETA, EPS)
            return
        L, n = self.orc, r1 - r0
        width = (NQ + 2 * NKV) * HD
        L.or_residual_rmsnorm(1, p(self.x, r0 * HIDDEN * 2), HIDDEN, p(self.d, r0 * HIDDEN * 2),
                              HIDDEN, p(self.y, r0 * HIDDEN * 2), HIDDEN, p(self.w), n, HIDDEN, EPS)
        L.or_qk_norm_rope(1, p(self.qkv, r0 * width * 2), p(self.qkv, (r0 * width + NQ * HD) * 2),
                          width, width, HD, HD, NQ, NKV, HD, HD, p(self.qw), p(self.kw),
                          p(self.pos, r0 * 4), n, THETA, EPS)
        L.or_silu_mul(1, p(self.h, r0 * INTER * 2), INTER, p(self.g, r0 * INTER * 2), INTER,
                      p(self.u, r0 * INTER * 2), INTER, n, INTER)

    def run(self, threads, rows_per_thread):
        ts = []
        for t in range(threads):
            r0 = (t * rows_per_thread) % self.rows
            r1 = min(r0 + rows_per_thread, self.rows)
            ts.append(threading.Thread(target=self.run_block, args=(r0, r1)))
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        return threads * rows_per_thread


def cpu_baseline(seconds=8.0):
    threads = host_threads()
    rpt = 8
    ch = CpuChain(max(threads * rpt, 64))
    ch.run(threads, 1)
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        done += ch.run(threads, rpt)
    el = time.perf_counter() - t0
    return {"value": round(done * B_ROW / el / 1e9, 3), "unit": "GB/s",
            "rows_per_s": round(done / el, 1), "cores": threads, "kind": ch.kind,
            "cpu": cpu_model(),
            "sample": f"{done} rows of the Qwen3-8B chain in {el:.1f} s on {threads} threads"}


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return
    threads = host_threads()
    ch = CpuChain(threads * 64)
    # size each step so the whole run stays within about 90 s
    t0 = time.perf_counter()
    ch.run(threads, 1)
    per_row = max(time.perf_counter() - t0, 1e-4)
    rpt = int(max(1, min(64, 90.0 / max(args.steps + args.warmup, 1) / per_row)))
    for _ in range(args.warmup):
        ch.run(threads, rpt)
    t0 = time.perf_counter()
    done = 0
    for _ in range(args.steps):
        done += ch.run(threads, rpt)
    el = time.perf_counter() - t0
    value = done * B_ROW / el / 1e9
    line = base_line(args, world, value, el * 1e3 / max(args.steps, 1))
    line["impl"] = "reference"
    line["rows_per_s"] = round(done / el, 1)
    line["cpu_baseline"] = {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                            "kind": ch.kind, "cpu": cpu_model(),
                            "sample": f"{threads * rpt} rows per step ({rpt} per thread)"}
    line["e2e"] = {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


def base_line(args, world, value, ms_per_step):
    return {
        "metric": "fused-layer-op HBM GB/s (% of B200 peak) and rows/s",
        "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "qwen3-8b-batched-prefill-layer-op-chain",
                   "rows_per_gpu": ROWS, "global_rows": ROWS * world, "hidden": HIDDEN,
                   "q_heads": NQ, "kv_heads": NKV, "head_dim": HD, "intermediate": INTER,
                   "bytes_per_row": B_ROW, "parallelism": f"rows{world}",
                   "l2": "inputs larger than L2 (x+d 512 MiB, q+k 256 MiB, gate+up 1.5 GiB)"},
    }


def read_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    (profiles/ncu_traffic.txt: `<kernel> <bytes_per_launch> <rows>` lines),
    scaled to the benchmark's row count, or None."""
    p = os.path.join(REPO, "profiles", "ncu_traffic.txt")
    try:
        with open(p) as f:
            for ln in f:
                parts = ln.split()
                if len(parts) >= 3 and parts[0] == kernel and not ln.startswith("#"):
                    return float(parts[1]) * ROWS / float(parts[2])
    except Exception:
        pass
    return None


def run_ours(args):
    import torch.distributed as dist
    rank, local, world = env_rank()
    torch, ane, rank, local = _setup_gpu(world)
    cur = torch.cuda.current_stream()
    row0, nrows = rank_rows(rank)
    b = make_chain_inputs(torch, nrows, HIDDEN, NQ, NKV, HD, INTER, SEQ, chain_seed(row0))
    chain = Chain(ane, b, ROWS, HIDDEN, NQ, NKV, HD, INTER, cur.cuda_stream)
    total_ms, per, clocks = time_device_chain(torch, dist, world, chain, args.steps,
                                              args.warmup, local)
    total_ms = max_over_ranks(torch, dist, world, total_ms)
    ms_step = total_ms / args.steps
    value = aggregate_gbs(world, nrows, ms_step)
    peak, peak_kind = measured_peak()
    names = ["residual_rmsnorm", "qk_norm_rope", "silu_mul"]
    bytes_k = [ROWS * B_NORM, ROWS * B_QK, ROWS * B_SILU]
    kern = {}
    for nm, ms, by in zip(names, per, bytes_k):
        kern[nm] = {"ms": round(ms, 5), "gb_s": round(by / ms / 1e6, 1),
                    "frac_of_peak": round(by / ms / 1e6 / peak, 4)}
    top = max(range(3), key=lambda i: per[i])
    top_gbs = bytes_k[top] / per[top] / 1e6
    traffic = read_traffic(names[top])
    del chain, b
    torch.cuda.empty_cache()

    e2e_steps = max(2, min(5, args.steps))
    if world > 1:
        dist.barrier()
    e_ms, h2d, d2h, e_launches = time_e2e_chain(torch, ane, ROWS, e2e_steps)
    e_ms = max_over_ranks(torch, dist, world, e_ms)
    e2e_val = aggregate_gbs(world, nrows, e_ms)
    torch.cuda.empty_cache()

    extras = time_extras(torch, ane) if (rank == 0 and not args.no_extras) else None
    cpu = cpu_baseline(args.cpu_seconds) if (rank == 0 and world == 1) else None
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = base_line(args, world, value, ms_step)
        line.update({
            "rows_per_s": round(world * ROWS / (ms_step * 1e-3), 1),
            "pct_of_hbm_peak": round(100 * value / world / peak, 2),
            "roofline": {"bound": "hbm", "kernel": names[top], "achieved": round(top_gbs, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(top_gbs / peak, 4),
                         "traffic": None if traffic is None else int(traffic),
                         "algorithmic_bytes": bytes_k[top]},
            "kernels": kern,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "ms_per_step": round(e_ms, 3),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "pinned host buffers, 8 row blocks over 2 streams"},
            "gpu_launches": 3 * args.steps,
            "clocks": clocks,
            "extra": extras,
        })
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ncu_case(cases, rows=16384):
    """Small cases for ncu captures: each kernel launched twice (a warm launch
    and the one to capture); inputs above L2, a few GB on the device."""
    import ctypes as C
    torch, ane, _, _ = _setup_gpu(1)
    L = ane.lib()
    cur = torch.cuda.current_stream()
    sp = C.c_void_p(cur.cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    if "chain" in cases:
        b = make_chain_inputs(torch, rows, HIDDEN, NQ, NKV, HD, INTER, SEQ, 1)
        ch = Chain(ane, b, rows, HIDDEN, NQ, NKV, HD, INTER, cur.cuda_stream)
        for _ in range(2):
            ch.launch()
            torch.cuda.synchronize()
        del b, ch
    if "convert" in cases:
        n = 1 << 29
        src = torch.randint(-32768, 32768, (n,), dtype=torch.int16, device="cuda")
        dst = torch.empty_like(src)
        for _ in range(2):
            assert L.ane_cuda_bf16_to_f16(P(dst), P(src), n, sp) == 0
        torch.cuda.synchronize()
        del src, dst
    if "sampler" in cases:
        r, v = 256, 151936
        g = torch.Generator(device="cuda").manual_seed(3)
        logits = torch.randn(r, v, device="cuda", generator=g) * 3
        hist = torch.randint(0, v, (r, 1024), device="cuda", dtype=torch.int32, generator=g)
        hlen = torch.full((r,), 1024, device="cuda", dtype=torch.int32)
        u = torch.rand(r, device="cuda", generator=g)
        tok = torch.empty(r, device="cuda", dtype=torch.int32)
        for _ in range(2):
            assert L.ane_cuda_sample_rows(P(logits), r, v, v, P(hist), P(hlen), 1024, P(u), 0.6,
                                          1.2, 256, 0.1, P(tok), sp) == 0
        torch.cuda.synchronize()
    if "attention" in cases:
        for B, H, hk, ln, dt in ((16, 32, 8, 4096, torch.float16), (1, 16, 8, 4096, torch.float32)):
            g = torch.Generator(device="cuda").manual_seed(9)
            q = torch.randn(B, H, 128, device="cuda", generator=g).to(dt)
            k = torch.randn(B, ln, hk, 128, device="cuda", generator=g).to(dt)
            v = torch.randn(B, ln, hk, 128, device="cuda", generator=g).to(dt)
            st = torch.full((B,), 1000, dtype=torch.int32, device="cuda")
            n = torch.full((B,), ln, dtype=torch.int32, device="cuda")
            for _ in range(2):
                ane.decode_attention(q, k, v, st, n, max_len=ln)
            torch.cuda.synchronize()
            del q, k, v
    if "pack" in cases:
        x = torch.randn(8192, 4096, device="cuda")
        surf = torch.zeros((256, 4096, 32), dtype=torch.int16, device="cuda")
        y = torch.empty_like(x)
        for _ in range(2):
            ane.ane_pack(x, surface=surf)
            ane.ane_unpack(surf, 8192, out=y)
        torch.cuda.synchronize()
        del x, surf, y
    print("ncu case done:", ",".join(sorted(cases)), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--ncu-case", default="",
                    help="comma list of chain,convert,sampler,attention,pack: run the small profiling "
                         "case and exit")
    args = ap.parse_args()
    if args.ncu_case:
        run_ncu_case(set(args.ncu_case.split(",")))
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
