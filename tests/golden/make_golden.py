"""Generates the golden fixtures in this directory from the REFERENCE's own
CPU code (core/cpu_ops.cpp, core/sampling.cpp, include/ane_lm/common.h,
core/safetensors.cpp), compiled by oracle/Makefile into
oracle/_ref/libaneref.so against the stand-in Accelerate headers.

Run from the repository root after `make -C oracle`:
    python tests/golden/make_golden.py

Inputs are seeded numpy draws stored in the fixtures themselves, so the
tests need neither the reference tree nor the same random streams.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from oracle_lib import load_ref  # noqa: E402


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def main():
    ref = load_ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libaneref.so is missing: run `make -C oracle` with the "
                         "reference tree present")

    # 1. BF16 -> FP16, every input
    a = np.arange(65536, dtype=np.uint16)
    out = np.empty_like(a)
    ref.ref_bf16_to_f16_vec(ptr(out), ptr(a), a.size)
    np.savez_compressed(os.path.join(HERE, "bf16_to_f16.npz"), bf16=a, f16=out)

    rng = np.random.default_rng(1234)

    # 2. rmsnorm rows (fp32, the reference's own precision)
    cases = {}
    for dim in (128, 1024, 2048, 4096, 1000):
        x = rng.standard_normal((4, dim)).astype(np.float32)
        x[0, :7] *= 50.0
        w = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
        y = np.empty_like(x)
        for r in range(x.shape[0]):
            ref.ref_rmsnorm(ptr(y[r]), ptr(x[r]), ptr(w), dim, np.float32(1e-6))
        cases[f"x_{dim}"], cases[f"w_{dim}"], cases[f"y_{dim}"] = x, w, y
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), **cases)

    # 3. per-head rmsnorm + RoPE with the model's cos/sin table (libm powf/cosf/sinf)
    nq, nkv, hd, theta = 16, 8, 128, 1e6
    positions = np.array([0, 1, 7, 511, 2047, 4095, 16383, 100000], np.int32)
    qk_in = rng.standard_normal((positions.size, nq + nkv, hd)).astype(np.float32)
    qw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    qk_out = qk_in.copy()
    cos = np.empty((positions.size, hd // 2), np.float32)
    sin = np.empty_like(cos)
    for i, pos in enumerate(positions):
        v = qk_out[i]
        for h in range(nq + nkv):
            ref.ref_rmsnorm(ptr(v[h]), ptr(v[h]), ptr(qw if h < nq else kw), hd, np.float32(1e-6))
        ref.ref_rope_row(ptr(cos[i]), ptr(sin[i]), int(pos), hd, np.float32(theta))
        ref.ref_apply_rope_cached(ptr(v), C.c_void_p(v.ctypes.data + nq * hd * 4), nq, nkv, hd,
                                  hd, hd, hd, int(pos), np.float32(theta), ptr(cos[i]),
                                  ptr(sin[i]))
    np.savez_compressed(os.path.join(HERE, "qk_rope.npz"), qk_in=qk_in, qk_out=qk_out, qw=qw,
                        kw=kw, positions=positions, cos=cos, sin=sin,
                        shape=np.array([nq, nkv, hd]), theta=np.float32(theta))

    # 4. silu_vec_inplace
    g = (rng.standard_normal(4096) * 4).astype(np.float32)
    g[:6] = [0.0, -0.0, -100.0, 100.0, -88.0, 250.0]
    s = g.copy()
    ref.ref_silu_vec_inplace(ptr(s), s.size)
    np.savez_compressed(os.path.join(HERE, "silu.npz"), x=g, y=s)

    # 5. sample_token: tokens and the (float)drand48() draw each used
    vocab = 4096
    rows = []
    for i in range(12):
        lg = (rng.standard_normal(vocab) * 3).astype(np.float32)
        hl = [0, 5, 300, 1024][i % 4]
        hist = rng.integers(-3, vocab + 3, size=max(hl, 1)).astype(np.int32)
        if hl > 10:
            hist[:40] = hist[0]  # repeated ids
        temp = [0.6, 0.0, 1.0, 0.6][i % 4] if i < 8 else 0.6
        rep = 1.2 if i % 3 else 1.0
        seed = 1000 + i
        u = C.c_float()
        tok = ref.ref_sample_token(ptr(lg), vocab, np.float32(temp), np.float32(rep), 256,
                                   np.float32(0.1), ptr(hist), hl, seed, C.byref(u))
        rows.append((lg, hist, hl, temp, rep, u.value, tok))
    hmax = max(r[1].size for r in rows)
    hist_m = np.full((len(rows), hmax), -1, np.int32)
    for i, r in enumerate(rows):
        hist_m[i, :r[1].size] = r[1]
    np.savez_compressed(
        os.path.join(HERE, "sampler.npz"),
        logits=np.stack([r[0] for r in rows]), history=hist_m,
        history_len=np.array([r[2] for r in rows], np.int32),
        temperature=np.array([r[3] for r in rows], np.float32),
        rep=np.array([r[4] for r in rows], np.float32),
        uniforms=np.array([r[5] for r in rows], np.float32),
        tokens=np.array([r[6] for r in rows], np.int32))

    # 6. `convert` of a small safetensors file: the reference writer's blob bytes
    with tempfile.TemporaryDirectory() as td:
        names = ["model.embed_tokens.weight", "model.layers.0.mlp.gate_proj.weight",
                 "model.norm.weight"]
        shapes = [(16, 8), (4, 8), (8,)]
        blobs = []
        header = {}
        off = 0
        for n, shp in zip(names, shapes):
            raw = rng.integers(0, 65536, size=int(np.prod(shp)), dtype=np.uint16)
            blobs.append(raw)
            header[n] = (shp, off, off + raw.nbytes)
            off += raw.nbytes
        f32 = np.arange(4, dtype=np.float32)
        header["extra.f32"] = ((4,), off, off + f32.nbytes)
        import json
        js = json.dumps({"__metadata__": {"format": "pt"}, **{
            k: {"dtype": "F32" if k == "extra.f32" else "BF16", "shape": list(v[0]),
                "data_offsets": [v[1], v[2]]} for k, v in header.items()}})
        path = os.path.join(td, "model.safetensors")
        with open(path, "wb") as fh:
            fh.write(struct.pack("<Q", len(js)))
            fh.write(js.encode())
            for b in blobs:
                fh.write(b.tobytes())
            fh.write(f32.tobytes())
        outdir = os.path.join(td, "ane_weights")
        os.makedirs(outdir)
        n = ref.ref_write_ane_blobs(path.encode(), outdir.encode())
        assert n == 3, n
        files = {}
        for n_ in names:
            rel = n_.replace(".", "/") + ".bin"
            files[n_] = np.frombuffer(open(os.path.join(outdir, rel), "rb").read(), np.uint8)
        np.savez_compressed(os.path.join(HERE, "convert_blobs.npz"),
                            safetensors=np.frombuffer(open(path, "rb").read(), np.uint8),
                            **{"blob:" + k: v for k, v in files.items()})
    # Fixtures of the next rows, from their own random stream so the ones
    # above stay as they were.
    rng2 = np.random.default_rng(4321)

    # 7. gqa_attention (core/cpu_ops.cpp:173-240) over rings, fp32 (inputs on
    #    a 1/64 grid, exact in fp16, stored as fp16 so the fixture stays
    #    small; the arithmetic is full fp32)
    att = {}
    q64 = lambda shape: (np.round(rng2.standard_normal(shape) * 64) / 64).astype(np.float32)  # noqa: E731
    for i, (H, hk, hd, cap, start, ln) in enumerate([(8, 2, 128, 256, 250, 256),
                                                     (32, 8, 128, 70, 60, 69),
                                                     (16, 4, 128, 200, 150, 190),
                                                     (16, 8, 128, 64, 7, 1),
                                                     (8, 8, 64, 100, 99, 37)]):
        q, k, v = q64((H, hd)), q64((cap, hk, hd)), q64((cap, hk, hd))
        o = np.empty((H, hd), np.float32)
        ref.ref_gqa_attention(ptr(o), ptr(q), ptr(k), ptr(v), H, hk, hd, hd, start, ln, cap)
        att.update({f"q{i}": q.astype(np.float16), f"k{i}": k.astype(np.float16),
                    f"v{i}": v.astype(np.float16), f"out{i}": o,
                    f"ring{i}": np.array([start, ln, cap], np.int32)})
    np.savez_compressed(os.path.join(HERE, "gqa_attention.npz"), **att)

    # 8. rmsnorm_gated (:33-39) and l2_normalize (:106-111), fp32 rows of 128
    x = (rng2.standard_normal((16, 128)) * 2).astype(np.float32)
    z = (rng2.standard_normal((16, 128)) * 4).astype(np.float32)
    z[0, :3] = [-90.0, 90.0, 40.0]
    w = (1.0 + 0.1 * rng2.standard_normal(128)).astype(np.float32)
    gated = np.empty_like(x)
    l2 = x.copy()
    for r in range(x.shape[0]):
        ref.ref_rmsnorm_gated(ptr(gated[r]), ptr(x[r]), ptr(z[r]), ptr(w), 128)
        ref.ref_l2_normalize(ptr(l2[r]), 128)
    np.savez_compressed(os.path.join(HERE, "hybrid_rows.npz"), x=x, z=z, w=w, gated=gated, l2=l2)

    # 9. the ANE-boundary conversions of the x86 branch (common.h:35-71):
    #    f32 -> f16 by truncation over random bit patterns and specials,
    #    f16 -> f32 over every half
    f32 = rng2.integers(0, 1 << 32, 8192, dtype=np.uint64).astype(np.uint32)
    f32[:8] = [0x7F800000, 0xFF800000, 0x7FC00000, 0x33000001, 0x387FC000, 0x477FF000, 0x1, 0x3F801000]
    f32 = f32.view(np.float32)
    trunc = np.empty(f32.size, np.uint16)
    ref.ref_f32_to_f16_vec(ptr(trunc), ptr(f32), f32.size)
    h = np.arange(65536, dtype=np.uint16)
    widen = np.empty(h.size, np.float32)
    ref.ref_f16_to_f32_vec(ptr(widen), ptr(h), h.size)
    np.savez_compressed(os.path.join(HERE, "ane_convert.npz"), f32=f32, trunc=trunc, widen=widen)

    # 10. load_bf16_to_f32 and the (1 + w) load_norm_weight (safetensors.cpp:264-306)
    b = rng2.integers(0, 65536, 2048, dtype=np.uint64).astype(np.uint16)
    b[:5] = [0x7F80, 0xFF80, 0x7FC1, 0x8000, 0x3F80]
    with tempfile.TemporaryDirectory() as td:
        import json
        js = json.dumps({"model.norm.weight": {"dtype": "BF16", "shape": [2048],
                                               "data_offsets": [0, 4096]}})
        path = os.path.join(td, "w.safetensors")
        with open(path, "wb") as fh:
            fh.write(struct.pack("<Q", len(js)))
            fh.write(js.encode())
            fh.write(b.tobytes())
        plain = np.empty(2048, np.float32)
        norm = np.empty(2048, np.float32)
        assert ref.ref_load_weight(path.encode(), b"model.norm.weight", 2048, 0, ptr(plain)) == 0
        assert ref.ref_load_weight(path.encode(), b"model.norm.weight", 2048, 1, ptr(norm)) == 0
    np.savez_compressed(os.path.join(HERE, "norm_weight.npz"), bf16=b, plain=plain, norm=norm)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
