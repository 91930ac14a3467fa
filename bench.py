"""Benchmark of the ANE-LM layer-op hot path on B200.

Headline (BASELINE metric "fused-layer-op HBM GB/s (% of B200 peak) and
rows/s at 1/2/4/8 GPUs"): the Qwen3-8B batched-prefill layer-op chain --
residual add + RMSNorm, per-head QK-norm + RoPE, SiLU-gate -- over a fixed
global batch of 64 x 512 = 32768 rows, partitioned by rows across the N GPUs
(strong scaling: rank r owns the contiguous block [r*32768/N, (r+1)*32768/N),
no collective on the data path).  A step is one pass of the three kernels
over each rank's rows.  Synthetic fp16 ~N(0,1) activations with 0.1% of
entries x50, each 512-row sequence generated from its own seed (so the
global inputs are the same at every N), positions row mod 512.  Each rank
rotates through enough buffer sets that a kernel's inputs were last touched
more than 1 GiB of traffic earlier (the L2 is 126 MB).

The same line carries the other BASELINE configs: the 256-row sampler and
the 8.19 B-parameter BF16->FP16 convert, both sharded over the N GPUs and
timed as the max over ranks, and (rank 0, one GPU) the Qwen3-1.7B prefill
chain, the Qwen3-0.6B batch-1 decode chain, decode attention and the ANE
packing.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line.  --impl reference times the reference's own CPU
code for the same chain (oracle/_ref, the reference sources compiled here;
the C restatement when that build is absent) on the host cores.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import math
import os
import subprocess
import sys
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
# each timed kernel's inputs must have been last touched at least this many
# bytes of traffic earlier (8x the 126 MB L2)
ROTATE_BYTES = 1 << 30
# sampler
S_ROWS, VOCAB, S_HIST = 256, 151936, 1024
B_SAMPLE_ROW = VOCAB * 4 + S_HIST * 4 + 4 + 4
# convert: embedding + 36 layers (q, k, v, o, gate, up,
# down) + lm_head, 4 bytes of traffic per parameter
CONVERT_PARAMS = 151936 * 4096 * 2 + 36 * (4096 * 4096 * 2 + 1024 * 4096 * 2 + 12288 * 4096 * 3)


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


def rank_rows(rank, world, total=ROWS):
    """Row sharding: the `total` global rows are split into `world`
    contiguous blocks whose sizes differ by at most one; rank r owns
    [r*total//world, (r+1)*total//world).  Returns (first row, row count).
    Rows are independent, so nothing crosses ranks on the data path."""
    r0 = rank * total // world
    return r0, (rank + 1) * total // world - r0


def seq_seed(s):
    """Seed of global sequence s (rows [s*SEQ, (s+1)*SEQ)) of the synthetic batch."""
    return 1234 + s


def aggregate_gbs(global_rows, ms):
    """Whole-job GB/s of the chain: all ranks' rows over the slowest rank's time."""
    return global_rows * B_ROW / (ms * 1e-3) / 1e9


def rotation_sets(set_bytes, min_bytes=ROTATE_BYTES):
    """How many copies of a buffer set the timed loop cycles through so that a
    kernel's inputs were last touched at least `min_bytes` earlier."""
    return max(1, math.ceil(min_bytes / max(set_bytes, 1)))


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
    """SM clock and throttle reasons sampled DURING the timed region.

    A thread reads NVML (the library nvidia-smi reports from) every ~2 ms
    from the moment the region starts until it ends, so that a region of a
    few milliseconds -- the multi-GPU steps -- still gets samples; without
    NVML bindings an `nvidia-smi -lms 100` process is the fallback, waited
    for until it prints before the region starts."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40),
               ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_s: float = 0.002, pci_bus_id: str | None = None):
        self.gpu = gpu_index
        self.pci = pci_bus_id  # NVML is matched by PCI address when given (device
        #                         numbering may differ from CUDA's)
        self.period = period_s
        self.samples = []  # (sm MHz, reason bits)
        self.max_mhz = None
        self.source = None
        self._nvml = None
        self._thread = None
        self._stop = None
        self.proc = None
        self.out = ""

    def _start_nvml(self):
        try:
            import threading

            import pynvml
            pynvml.nvmlInit()
            h = None
            if self.pci:
                try:
                    h = pynvml.nvmlDeviceGetHandleByPciBusId(self.pci.encode())
                except Exception:
                    h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            sample = lambda: (float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),  # noqa: E731
                              int(reasons(h)))
            sample()
        except Exception:
            return False
        self._nvml = pynvml
        self._stop = threading.Event()

        def run():
            while True:
                try:
                    self.samples.append(sample())
                except Exception:
                    pass
                if self._stop.wait(self.period):
                    break

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        self.source = "nvml, every 2 ms"
        return True

    def __enter__(self):
        if self._start_nvml():
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            first = self.proc.stdout.readline()  # sampling has begun
            self.out = first
            self.source = "nvidia-smi, every 100 ms"
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                rest, _ = self.proc.communicate(timeout=5)
                self.out += rest
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        sms, reasons = [], set()
        if self.source and self.source.startswith("nvml"):
            for mhz, bits in self.samples:
                sms.append(mhz)
                reasons.update(nm for nm, b in self.REASONS if bits & b)
        else:
            names = [nm for nm, _ in self.REASONS]
            for ln in (self.out or "").splitlines():
                parts = [p.strip() for p in ln.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sms.append(float(parts[1]))
                    self.max_mhz = float(parts[2])
                except ValueError:
                    continue
                for nm, v in zip(names, parts[5:9]):
                    if v.lower() in ("active", "1"):
                        reasons.add(nm)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": self.source}
        sms.sort()
        return {"sm_mhz": sms[len(sms) // 2], "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(sms), "source": self.source}


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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    sys.path.insert(0, PKG)
    import ane_lm_cuda
    ane_lm_cuda.lib()  # fails loudly when the library is missing
    return torch, ane_lm_cuda, rank, local


def parse_cpulist(text):
    """The CPU set of a Linux cpulist string ("0-3,8,10-11")."""
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def pci_address(torch, dev):
    """The PCI address ("0000:1b:00.0") of CUDA device `dev`, or None."""
    try:
        p = torch.cuda.get_device_properties(dev)
        return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    except (AttributeError, RuntimeError, AssertionError, TypeError, ValueError):
        return None


def bind_near_gpu(torch, dev, sysfs="/sys/bus/pci/devices"):
    """Keep this process on the host CPUs next to GPU `dev` (its PCI
    device's local_cpulist), so that the pinned host buffers it allocates
    afterwards are placed on that NUMA node by first touch and the
    host<->device copies of one rank do not cross the socket interconnect.
    Returns the cpulist applied, or None when there is nothing to narrow
    (one NUMA node, or the topology is not visible)."""
    pid = pci_address(torch, dev)
    if pid is None:
        return None
    try:
        with open(os.path.join(sysfs, pid, "local_cpulist")) as f:
            text = f.read().strip()
        want = parse_cpulist(text) & os.sched_getaffinity(0)
    except (OSError, AttributeError, ValueError):
        return None
    if not want or want == os.sched_getaffinity(0):
        return None
    os.sched_setaffinity(0, want)
    return text


def make_chain_inputs(torch, row0, rows, hidden, nq, nkv, hd, inter, seq, device="cuda"):
    """Rows [row0, row0 + rows) of the global synthetic batch: fp16 ~N(0,1)
    with 0.1% of entries x50, positions (global row) mod seq.  Every
    sequence of `seq` rows comes from its own seed (`seq_seed`), so a row's
    values do not depend on how the batch is split across ranks.  The norm
    weights come from one fixed seed."""
    width = (nq + 2 * nkv) * hd
    cols = {"x": hidden, "d": hidden, "qkv": width, "gate": inter, "up": inter}
    parts = {k: [] for k in cols}
    for s in range(row0 // seq, (row0 + rows + seq - 1) // seq):
        g = torch.Generator(device=device).manual_seed(seq_seed(s))
        lo, hi = max(row0, s * seq) - s * seq, min(row0 + rows, (s + 1) * seq) - s * seq
        for k, n in cols.items():
            a = torch.randn(seq, n, device=device, generator=g, dtype=torch.float32)
            m = torch.rand(seq, n, device=device, generator=g) < 1e-3
            a[m] *= 50.0
            parts[k].append(a[lo:hi].half())
    b = {k: torch.cat(v) if len(v) > 1 else v[0].contiguous() for k, v in parts.items()}
    gw = torch.Generator(device=device).manual_seed(99)
    b["w"] = (1 + 0.1 * torch.randn(hidden, device=device, generator=gw)).float()
    b["qw"] = (1 + 0.1 * torch.randn(hd, device=device, generator=gw)).float()
    b["kw"] = (1 + 0.1 * torch.randn(hd, device=device, generator=gw)).float()
    b["pos"] = ((row0 + torch.arange(rows, device=device, dtype=torch.int64)) % seq).to(torch.int32)
    b["y"] = torch.empty(rows, hidden, device=device, dtype=torch.float16)
    b["h"] = torch.empty(rows, inter, device=device, dtype=torch.float16)
    return b


def chain_set_bytes(rows, hidden, nq, nkv, hd, inter):
    """Device bytes of one buffer set: x, d, y, the qkv rows, gate, up, h (fp16)."""
    return rows * (3 * hidden + (nq + 2 * nkv) * hd + 3 * inter) * 2


def clone_set(torch, b):
    return {k: v.clone() for k, v in b.items()}


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


EVENT_EVERY = 4  # per-kernel events on one timed step in this many


def instrumented(i, steps):
    """Whether timed step i carries per-kernel events: every EVENT_EVERY-th
    step (the last one when there are fewer).  An event recorded between two
    kernels ends the programmatic overlap of their launches, so events on
    every step would slow the chain they measure (about 14% at 4,096 rows
    per GPU)."""
    return i % EVENT_EVERY == EVENT_EVERY - 1 or (steps < EVENT_EVERY and i == steps - 1)


def time_device_chain(torch, dist, world, chains, steps, warmup, gpu_index):
    """K steps over the rank's rows; step i uses buffer set i mod len(chains).
    Returns the K steps' time, each kernel's mean duration over the
    instrumented steps, and the clock record."""
    n = len(chains)
    for i in range(warmup):
        chains[i % n].launch()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] if instrumented(i, steps)
           else None for i in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(gpu_index, pci_bus_id=pci_address(torch, gpu_index)) as clk:
        start.record()
        for i in range(steps):
            chains[i % n].launch(evs[i])
        end.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    total_ms = start.elapsed_time(end)
    timed = [e for e in evs if e is not None]
    per = [sum(e[k].elapsed_time(e[k + 1]) for e in timed) / len(timed) for k in range(3)]
    return total_ms, per, clk.summary()


def max_over_ranks(torch, dist, world, v):
    """The slowest rank's value(s): a MAX all-reduce of one number or a list
    (the timing collective, never on the data path); on gloo too."""
    if world == 1:
        return v
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    vals = list(v) if isinstance(v, (list, tuple)) else [v]
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    out = [float(a) for a in t.tolist()]
    return out if isinstance(v, (list, tuple)) else out[0]


def time_e2e_chain(torch, ane, rows, steps, chunks=16):
    """The same chain through the public C ABI with HOST buffers: every step
    copies its inputs (x, d, the q and k heads, gate, up) from pinned memory
    to the device, runs the three kernels and copies the outputs (x, y, the
    q and k heads, h) back, in `chunks` row blocks over two streams so copies
    overlap the kernels.  The v heads of a qkv row are neither read nor
    written by the chain, so the host keeps the q and k heads of each row
    (n_q + n_kv heads) and moves only those."""
    import ctypes as C
    L = ane.lib()
    width = (NQ + NKV) * HD  # q and k heads
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
    bounds = [c * rows // chunks for c in range(chunks + 1)]
    cmax = max(bounds[c + 1] - bounds[c] for c in range(chunks))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    dev = [{k: torch.empty(cmax, n, device="cuda", dtype=torch.float16)
            for k, n in (("x", HIDDEN), ("d", HIDDEN), ("y", HIDDEN), ("q", width),
                         ("g", INTER), ("u", INTER), ("h", INTER))} for _ in streams]
    P = lambda t, off=0: C.c_void_p(t.data_ptr() + off)  # noqa: E731

    def step():
        for c in range(chunks):
            s = streams[c % 2]
            b = dev[c % 2]
            r0, r1 = bounds[c], bounds[c + 1]
            cr = r1 - r0
            if cr == 0:
                continue
            with torch.cuda.stream(s):
                b["x"][:cr].copy_(hx[r0:r1], non_blocking=True)
                b["d"][:cr].copy_(hd_[r0:r1], non_blocking=True)
                b["q"][:cr].copy_(hq[r0:r1], non_blocking=True)
                b["g"][:cr].copy_(hg[r0:r1], non_blocking=True)
                b["u"][:cr].copy_(hu[r0:r1], non_blocking=True)
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
                hx[r0:r1].copy_(b["x"][:cr], non_blocking=True)
                oy[r0:r1].copy_(b["y"][:cr], non_blocking=True)
                hq[r0:r1].copy_(b["q"][:cr], non_blocking=True)
                oh[r0:r1].copy_(b["h"][:cr], non_blocking=True)

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


def _timed(torch, fn, n):
    fn(0)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(n):
        fn(i)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def _barrier(dist, world):
    if world > 1:
        dist.barrier()


def time_sharded_extras(torch, dist, ane, rank, world, reps=20):
    """BASELINE configs 4 and 5, partitioned like the chain: the 256 sampler
    rows split 256/N per rank, the 8.19 B convert parameters split by
    elements; each timed as the slowest rank's mean launch time.  Inputs
    rotate through copies larger than L2 in total."""
    import ctypes as C
    L = ane.lib()
    out = {}
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t, off=0: C.c_void_p(t.data_ptr() + off)  # noqa: E731

    # sampler: rank's rows of 256 x 151936; row j's inputs from seed 3 + j
    r0, n = rank_rows(rank, world, S_ROWS)
    rows = max(n, 1)
    logits = torch.empty(rows, VOCAB, device="cuda")
    hist = torch.empty(rows, S_HIST, device="cuda", dtype=torch.int32)
    u = torch.empty(rows, device="cuda")
    for j in range(n):
        g = torch.Generator(device="cuda").manual_seed(3 + r0 + j)
        logits[j] = torch.randn(VOCAB, device="cuda", generator=g) * 3
        hist[j] = torch.randint(0, VOCAB, (S_HIST,), device="cuda", dtype=torch.int32, generator=g)
        u[j] = torch.rand(1, device="cuda", generator=g)
    hlen = torch.full((rows,), S_HIST, device="cuda", dtype=torch.int32)
    tok = torch.empty(rows, device="cuda", dtype=torch.int32)
    nset = rotation_sets(rows * VOCAB * 4, 512 << 20)
    lsets = [logits] + [logits.clone() for _ in range(nset - 1)]
    _barrier(dist, world)
    ms = _timed(torch, lambda i: L.ane_cuda_sample_rows(
        P(lsets[i % nset]), n, VOCAB, VOCAB, P(hist), P(hlen), S_HIST, P(u), 0.6, 1.2, 256, 0.1,
        P(tok), sp), max(reps, nset)) if n else 0.0
    ms = max_over_ranks(torch, dist, world, ms)
    out["sampler_256x151936"] = {
        "rows": S_ROWS, "rows_per_gpu": -(-S_ROWS // world), "ms": round(ms, 4),
        "rows_per_s": round(S_ROWS / ms * 1e3, 1),
        "gb_s": round(S_ROWS * B_SAMPLE_ROW / ms / 1e6, 1),
        "l2": f"{nset} rotating logits copies per GPU"}
    del lsets, logits, hist, u, tok, hlen
    torch.cuda.empty_cache()

    # convert: the rank's element range of the flat 8.19 B-parameter checkpoint
    e0, ne = rank_rows(rank, world, CONVERT_PARAMS)
    src = torch.randint(-32768, 32768, (ne,), dtype=torch.int16, device="cuda")
    dst = torch.empty_like(src)
    _barrier(dist, world)
    ms = _timed(torch, lambda i: L.ane_cuda_bf16_to_f16(P(dst), P(src), ne, sp), reps)
    ms = max_over_ranks(torch, dist, world, ms)
    out["convert_qwen3_8b"] = {"params": CONVERT_PARAMS, "params_per_gpu": -(-CONVERT_PARAMS // world),
                               "ms": round(ms, 4),
                               "gb_s": round(CONVERT_PARAMS * 4 / ms / 1e6, 1),
                               "params_per_s": round(CONVERT_PARAMS / ms * 1e3, 1)}
    del src, dst
    torch.cuda.empty_cache()
    return out


def time_single_gpu_extras(torch, ane, reps=20):
    """The single-GPU configs: the Qwen3-1.7B prefill chain, the Qwen3-0.6B
    batch-1 decode chain latency, decode attention and the ANE-boundary
    packing."""
    import ctypes as C
    L = ane.lib()
    out = {}
    cur = torch.cuda.current_stream()
    P = lambda t, off=0: C.c_void_p(t.data_ptr() + off)  # noqa: E731
    peak, _ = measured_peak()

    # Qwen3-1.7B prefill chain, T = 2048 (226 MB of buffers: rotated copies)
    shape = (2048, 16, 8, 128, 6144)
    b = make_chain_inputs(torch, 0, 2048, 2048, *shape[1:], 2048)
    nset = rotation_sets(chain_set_bytes(2048, 2048, *shape[1:]))
    sets = [b] + [clone_set(torch, b) for _ in range(nset - 1)]
    chs = [Chain(ane, s, 2048, 2048, *shape[1:], cur.cuda_stream) for s in sets]
    ms = _timed(torch, lambda i: chs[i % nset].launch(), reps * 5)
    out["prefill_qwen3_1p7b_t2048"] = {"ms": round(ms, 4),
                                       "gb_s": round(2048 * 65536 / ms / 1e6, 1),
                                       "frac_of_peak": round(2048 * 65536 / ms / 1e6 / peak, 4),
                                       "l2": f"{nset} rotating buffer sets"}
    del b, sets, chs

    # Qwen3-0.6B decode, batch 1: gather (fp16 table -> fp32 row) fused with
    # the residual add + RMSNorm that reads it, QK-norm+RoPE and SiLU-gate in
    # fp32, replayed as one CUDA graph
    g = torch.Generator(device="cuda").manual_seed(3)
    table = (torch.randn(151936, 1024, device="cuda", generator=g) * 0.02).half()
    tid = torch.randint(0, 151936, (1,), device="cuda", dtype=torch.int32, generator=g)
    x = torch.randn(1, 1024, device="cuda", generator=g)
    y = torch.empty_like(x)
    w = torch.ones(1024, device="cuda")
    qkv = torch.randn(1, (16 + 16) * 128, device="cuda", generator=g)
    pos = torch.randint(0, 4096, (1,), device="cuda", dtype=torch.int32, generator=g)
    ga, up, h = (torch.randn(1, 3072, device="cuda", generator=g) for _ in range(3))
    gs = torch.cuda.Stream()

    def decode(stream):
        s = C.c_void_p(stream.cuda_stream)
        st = L.ane_cuda_embedding_rmsnorm(0, P(x), 1024, P(y), 1024, P(table), 1, P(tid), 1, 151936,
                                          1024, 1, P(w), EPS, s)
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
    ms = _timed(torch, lambda i: graph.replay(), 200)
    del graph
    # the same step 16 times in one graph: the host's graph launches, which
    # the one-step replays above also measure, are amortised as they are in
    # a whole-model graph
    graph16 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph16, stream=gs):
        for _ in range(16):
            decode(gs)
    ms16 = _timed(torch, lambda i: graph16.replay(), 25) / 16
    del graph16
    out["decode_qwen3_0p6b_b1"] = {"us_per_token": round(ms * 1e3, 2),
                                   "us_per_step_in_16_step_graph": round(ms16 * 1e3, 2),
                                   "kernels": 3}

    # decode attention over the KV ring: Qwen3-0.6B batch 1 with the
    # reference's fp32 cache, and Qwen3-8B batch 64 with an fp16 cache; 4096
    # keys, ring start mid-cache (wrapped).  CUDA graph of back-to-back calls
    # over rotating cache copies (more than L2 in total).
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
    for name, fn in (("ane_pack_32k_x_4096", lambda i: ane.ane_pack(x, surface=surf)),
                     ("ane_unpack_32k_x_4096", lambda i: ane.ane_unpack(surf, T, out=y))):
        ms = _timed(torch, fn, reps)
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
# CPU: the reference's own code (oracle/_ref) or the C restatement
# ---------------------------------------------------------------------------
def _cpu_libs():
    sys.path.insert(0, os.path.join(REPO, "tests"))
    from oracle_lib import Oracle, load_ref
    ref = load_ref()
    return ref, ("reference" if ref is not None else "port"), (None if ref is not None
                                                               else Oracle().lib)


class CpuChain:
    """The layer-op chain of the reference over host buffers of the whole
    32,768-row batch (about 3.6 GB, far beyond the host's caches), streamed
    in order: each call takes the next `n` rows (cycling) and splits them
    into contiguous blocks over a pool of threads (ctypes releases the GIL,
    so the blocks run in parallel).  The buffers hold `distinct` seeded rows
    tiled over the batch."""

    def __init__(self, rows=ROWS, distinct=512):
        import numpy as np
        self.np = np
        self.ref, self.kind, self.orc = _cpu_libs()
        rng = np.random.default_rng(17)
        width = (NQ + 2 * NKV) * HD

        def act(n):
            a = rng.standard_normal((distinct, n), dtype=np.float32)
            a[rng.random((distinct, n)) < 1e-3] *= 50.0
            a = a.astype(np.float16)
            return np.ascontiguousarray(np.tile(a, (-(-rows // distinct), 1))[:rows])

        self.rows = rows
        self.x, self.d = act(HIDDEN), act(HIDDEN)
        self.y = np.empty_like(self.x)
        self.w = (1 + 0.1 * rng.standard_normal(HIDDEN)).astype(np.float32)
        self.qkv = act(width)
        self.qw = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
        self.kw = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32)
        self.pos = (np.arange(rows) % SEQ).astype(np.int32)
        self.g, self.u = act(INTER), act(INTER)
        self.h = np.empty_like(self.g)
        self.cursor = 0
        self.pool = cf.ThreadPoolExecutor(max_workers=host_threads())

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

    def run(self, threads, n):
        """The next n rows (n <= rows), split over `threads` threads; returns n."""
        spans = []
        for t in range(threads):
            a = self.cursor + t * n // threads
            b = self.cursor + (t + 1) * n // threads
            while a < b:  # split at the wrap-around of the row buffer
                lo = a % self.rows
                hi = min(lo + (b - a), self.rows)
                spans.append((lo, hi))
                a += hi - lo
        self.cursor = (self.cursor + n) % self.rows
        list(self.pool.map(lambda s: self.run_block(*s), spans))
        return n

    def stream_for(self, threads, seconds, rows_per_thread):
        """Rows per second over `seconds` of consecutive calls."""
        self.run(threads, threads)  # warm the code and the pool
        done, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            done += self.run(threads, threads * rows_per_thread)
        return done, time.perf_counter() - t0


def cpu_sampler_baseline(threads, seconds=2.0):
    """The reference's sample_token (core/sampling.cpp:10-66) on BASELINE
    config 4's rows (fp32 logits ~N(0,3), 1024-id histories, T 0.6, penalty
    1.2 over the last 256 ids, frequency 0.1), rows spread over `threads`
    threads.  sample_token draws from the process-wide drand48 state, which
    threads share without a lock: the draws may interleave, the work per
    row does not change (timing only)."""
    import ctypes as C
    import numpy as np
    ref, kind, orc = _cpu_libs()
    rng = np.random.default_rng(5)
    rows = S_ROWS
    logits = (rng.standard_normal((rows, VOCAB), dtype=np.float32) * 3).astype(np.float32)
    hist = rng.integers(0, VOCAB, size=(rows, S_HIST)).astype(np.int32)
    p = lambda a, off=0: C.c_void_p(a.ctypes.data + off)  # noqa: E731

    def one(i):
        j = i % rows
        if ref is not None:
            u = C.c_float()
            ref.ref_sample_token(p(logits, j * VOCAB * 4), VOCAB, 0.6, 1.2, 256, 0.1,
                                 p(hist, j * S_HIST * 4), S_HIST, 1000 + i, C.byref(u))
        else:
            uu = np.array([0.5], np.float32)
            hl = np.array([S_HIST], np.int32)
            tk = np.zeros(1, np.int32)
            orc.or_sample_rows(p(logits, j * VOCAB * 4), 1, VOCAB, VOCAB, p(hist, j * S_HIST * 4),
                               p(hl), S_HIST, p(uu), 0.6, 1.2, 256, 0.1, p(tk))

    out = {}
    with cf.ThreadPoolExecutor(max_workers=threads) as pool:
        for nthr in sorted({1, threads}):
            list(pool.map(one, range(nthr)))
            done, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < seconds:
                batch = nthr * 4
                if nthr == 1:
                    for i in range(batch):
                        one(done + i)
                else:
                    list(pool.map(one, range(done, done + batch)))
                done += batch
            el = time.perf_counter() - t0
            out["rows_per_s" if nthr == threads else "rows_per_s_1thread"] = round(done / el, 1)
    out.update({"kind": kind, "cores": threads,
                "gb_s": round(out["rows_per_s"] * B_SAMPLE_ROW / 1e9, 3),
                "ms_per_256_rows": round(S_ROWS / out["rows_per_s"] * 1e3, 2),
                "sample": f"rows of 256 x {VOCAB} logits for ~{seconds:.0f} s per thread count"})
    return out


def cpu_convert_baseline(threads, seconds=2.0, n=1 << 28):
    """The reference's bf16_to_f16_vec (include/ane_lm/common.h:73-83) on
    BASELINE config 5's values (bf16 of N(0,0.02) with 1e-4 of entries of
    magnitude 65536..1e6): 2^28 elements (512 MiB in, 512 MiB out), split
    over `threads` threads, streamed for ~`seconds`."""
    import ctypes as C
    import numpy as np
    ref, kind, orc = _cpu_libs()
    rng = np.random.default_rng(6)
    m = 1 << 22
    v = (rng.standard_normal(m, dtype=np.float32) * 0.02)
    big = rng.random(m) < 1e-4
    v[big] = np.sign(rng.standard_normal(big.sum())) * rng.uniform(65536, 1e6, big.sum())
    bf = (v.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    src = np.tile(bf, n // m)
    dst = np.empty_like(src)
    fn = ref.ref_bf16_to_f16_vec if ref is not None else orc.or_bf16_to_f16_vec
    out = {}
    with cf.ThreadPoolExecutor(max_workers=threads) as pool:
        for nthr in sorted({1, threads}):
            spans = [(t * n // nthr, (t + 1) * n // nthr) for t in range(nthr)]
            step = n if nthr > 1 else n // 8

            def conv(s):
                a, b = s
                fn(C.c_void_p(dst.ctypes.data + 2 * a), C.c_void_p(src.ctypes.data + 2 * a), b - a)

            done, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < seconds:
                if nthr > 1:
                    list(pool.map(conv, spans))
                else:
                    off = done % n
                    conv((off, off + step))
                done += step
            el = time.perf_counter() - t0
            key = "gb_s" if nthr == threads else "gb_s_1thread"
            out[key] = round(done * 4 / el / 1e9, 3)
    out.update({"kind": kind, "cores": threads,
                "ms_per_8p19b_params": round(CONVERT_PARAMS * 4 / (out["gb_s"] * 1e9) * 1e3, 1),
                "sample": f"{n} elements (512 MiB in, 512 MiB out), ~{seconds:.0f} s per thread count"})
    return out


def cpu_baseline(seconds=6.0):
    """The reference's chain on the host cores, streamed over the whole
    32,768-row batch: all threads (the `value`) and one thread; then the
    reference sampler (config 4) and convert (config 5) beside them."""
    threads = host_threads()
    ch = CpuChain(ROWS)
    done, el = ch.stream_for(threads, seconds, 64)
    done1, el1 = ch.stream_for(1, seconds / 2, 32)
    value = done * B_ROW / el / 1e9
    out = {"value": round(value, 3), "unit": "GB/s", "rows_per_s": round(done / el, 1),
           "cores": threads, "kind": ch.kind, "cpu": cpu_model(),
           "value_1thread": round(done1 * B_ROW / el1 / 1e9, 3),
           "rows_per_s_1thread": round(done1 / el1, 1),
           "sample": (f"{done} rows of the Qwen3-8B chain streamed through the 32,768-row batch "
                      f"in {el:.1f} s on {threads} threads; {done1} rows in {el1:.1f} s on 1 thread")}
    del ch
    out["sampler"] = cpu_sampler_baseline(threads)
    out["convert"] = cpu_convert_baseline(threads)
    return out


def run_reference(args):
    """The reference arm: the reference's own CPU chain (oracle/_ref) on all
    host threads, streamed over the 32,768-row batch, each step a bounded
    sample of it so the whole run stays within about 90 s.  Rank 0 alone
    runs it; the other ranks return at once."""
    rank, _, world = env_rank()
    if rank != 0:
        return
    threads = host_threads()
    ch = CpuChain(ROWS)
    ch.run(threads, threads)
    t0 = time.perf_counter()
    ch.run(threads, threads * 4)
    per_row = max((time.perf_counter() - t0) / (threads * 4), 1e-6)
    budget = 90.0 / max(args.steps + args.warmup, 1)
    n = int(max(threads, min(ROWS, budget / per_row)))
    for _ in range(args.warmup):
        ch.run(threads, n)
    t0 = time.perf_counter()
    done = 0
    for _ in range(args.steps):
        done += ch.run(threads, n)
    el = time.perf_counter() - t0
    value = done * B_ROW / el / 1e9
    line = base_line(args, world, value, el * 1e3 / max(args.steps, 1))
    line["impl"] = "reference"
    line["rows_per_s"] = round(done / el, 1)
    line["cpu_baseline"] = {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                            "kind": ch.kind, "cpu": cpu_model(),
                            "sample": f"{n} consecutive rows of the 32,768-row batch per step"}
    line["e2e"] = {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


def base_line(args, world, value, ms_per_step, l2_note=None):
    return {
        "metric": "fused-layer-op HBM GB/s (% of B200 peak) and rows/s at 1/2/4/8 GPUs",
        "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "qwen3-8b-batched-prefill-layer-op-chain",
                   "global_rows": ROWS, "rows_per_gpu": -(-ROWS // world), "sequences": ROWS // SEQ,
                   "seq_len": SEQ, "hidden": HIDDEN, "q_heads": NQ, "kv_heads": NKV,
                   "head_dim": HD, "intermediate": INTER, "bytes_per_row": B_ROW,
                   "parallelism": f"rows/{world}",
                   "l2": l2_note or "inputs larger than L2"},
    }


def read_traffic(kernel, rows):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    (profiles/ncu_traffic.txt: `<kernel> <bytes_per_launch> <rows>` lines),
    scaled to `rows`, or None."""
    p = os.path.join(REPO, "profiles", "ncu_traffic.txt")
    try:
        with open(p) as f:
            for ln in f:
                parts = ln.split()
                if len(parts) >= 3 and parts[0] == kernel and not ln.startswith("#"):
                    return float(parts[1]) * rows / float(parts[2])
    except Exception:
        pass
    return None


def run_ours(args):
    import torch.distributed as dist
    rank, local, world = env_rank()
    torch, ane, rank, local = _setup_gpu(world)
    cur = torch.cuda.current_stream()
    row0, nrows = rank_rows(rank, world)
    shape = (HIDDEN, NQ, NKV, HD, INTER)
    b = make_chain_inputs(torch, row0, nrows, *shape, SEQ)
    set_bytes = chain_set_bytes(nrows, *shape)
    nset = rotation_sets(set_bytes)
    sets = [b] + [clone_set(torch, b) for _ in range(nset - 1)]
    chains = [Chain(ane, s, nrows, *shape, cur.cuda_stream) for s in sets]
    # bytes streamed between two launches of one kernel on the same set
    reuse = nset * nrows * B_ROW - nrows * max(B_NORM, B_QK, B_SILU)
    l2_note = (f"{nset} rotating buffer set(s) of {set_bytes / 2**20:.0f} MiB per GPU: each "
               f"kernel's inputs were last touched >= {reuse / 2**20:.0f} MiB of traffic earlier "
               f"(L2 126 MB)")
    total_ms, per, clocks = time_device_chain(torch, dist, world, chains, args.steps,
                                              args.warmup, local)
    mx = max_over_ranks(torch, dist, world, [total_ms] + per)
    total_ms, per = mx[0], mx[1:]
    ms_step = total_ms / args.steps
    value = aggregate_gbs(ROWS, ms_step)
    peak, peak_kind = measured_peak()
    rows_gpu = -(-ROWS // world)  # the largest block: the slowest rank's rows
    names = ["residual_rmsnorm", "qk_norm_rope", "silu_mul"]
    bytes_k = [rows_gpu * B_NORM, rows_gpu * B_QK, rows_gpu * B_SILU]
    kern = {}
    for nm, ms, by in zip(names, per, bytes_k):
        kern[nm] = {"ms": round(ms, 5), "gb_s": round(by / ms / 1e6, 1),
                    "frac_of_peak": round(by / ms / 1e6 / peak, 4)}
    top = max(range(3), key=lambda i: per[i])
    top_gbs = bytes_k[top] / per[top] / 1e6
    traffic = read_traffic(names[top], rows_gpu)
    del chains, sets, b
    torch.cuda.empty_cache()

    e2e_steps = max(2, min(5, args.steps))
    # with several ranks on a multi-socket host, each rank's pinned buffers
    # and copies stay on its GPU's socket (the CPU baseline, rank 0 at N = 1,
    # keeps every host thread)
    bound = bind_near_gpu(torch, local) if world > 1 else None
    _barrier(dist, world)
    e_ms, h2d, d2h, e_launches = time_e2e_chain(torch, ane, nrows, e2e_steps)
    e_ms = max_over_ranks(torch, dist, world, e_ms)
    e2e_val = aggregate_gbs(ROWS, e_ms)
    torch.cuda.empty_cache()

    extras = None
    if not args.no_extras:
        extras = time_sharded_extras(torch, dist, ane, rank, world)
        if rank == 0:
            extras.update(time_single_gpu_extras(torch, ane))
    cpu = cpu_baseline(args.cpu_seconds) if (rank == 0 and world == 1) else None
    _barrier(dist, world)
    if rank == 0:
        line = base_line(args, world, value, ms_step, l2_note)
        line.update({
            "rows_per_s": round(ROWS / (ms_step * 1e-3), 1),
            "pct_of_hbm_peak": round(100 * value / world / peak, 2),
            "per_gpu_gb_s": round(value / world, 1),
            "roofline": {"bound": "hbm", "kernel": names[top], "achieved": round(top_gbs, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(top_gbs / peak, 4),
                         "traffic": None if traffic is None else int(traffic),
                         "algorithmic_bytes": bytes_k[top]},
            "kernels": kern,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "ms_per_step": round(e_ms, 3),
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "note": "pinned host buffers, each rank its own rows in 16 blocks over 2 streams"
                            + (f"; rank 0 bound to CPUs {bound} (its GPU's NUMA node)" if bound else "")},
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
    # chain: 16,384 rows (several waves of CTAs); chain_small: 4,096 rows,
    # the rows per GPU at eight GPUs, where the row kernels take their
    # one-wave forms (RMSNorm with d in shared memory, QK-norm with two
    # iterations of loads in flight)
    for case, n in (("chain", rows), ("chain_small", ROWS // 8)):
        if case not in cases:
            continue
        b = make_chain_inputs(torch, 0, n, HIDDEN, NQ, NKV, HD, INTER, SEQ)
        ch = Chain(ane, b, n, HIDDEN, NQ, NKV, HD, INTER, cur.cuda_stream)
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
    attn = []
    if "attention" in cases or "attn_f16" in cases:
        attn.append((16, 32, 8, 4096, torch.float16))
    if "attention" in cases or "attn_f32" in cases:
        attn.append((1, 16, 8, 4096, torch.float32))
    if attn:
        for B, H, hk, ln, dt in attn:
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
    if "embed" in cases:
        # the decode step's first RMSNorm fed by the embedding gather, at prefill rows
        g = torch.Generator(device="cuda").manual_seed(5)
        table = (torch.randn(VOCAB, HIDDEN, device="cuda", generator=g) * 0.05).half()
        ids = torch.randint(0, VOCAB, (rows,), device="cuda", dtype=torch.int32, generator=g)
        w = torch.rand(HIDDEN, device="cuda", generator=g) + 0.5
        x = torch.empty(rows, HIDDEN, dtype=torch.float16, device="cuda")
        out = torch.empty_like(x)
        for _ in range(2):
            ane.embedding_rmsnorm(table, ids, w, x=x, out=out)
        torch.cuda.synchronize()
        del table, x, out
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
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=6.0)
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--ncu-case", default="",
                    help="comma list of chain,chain_small,convert,sampler,attention (attn_f16, attn_f32),embed,pack: "
                         "run the small profiling case and exit")
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
