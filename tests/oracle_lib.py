"""ctypes bindings to the test oracle (oracle/liboracle.so) and to the
reference sources compiled with the shim (oracle/_ref/libaneref.so).

Test infrastructure: only tests, ``__graft_entry__.smoke`` and the CPU
baseline leg of ``bench.py`` use this module, and only as the checker.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(REPO, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "liboracle.so")
REF_SO = os.path.join(ORACLE_DIR, "_ref", "libaneref.so")

F32, F16, BF16 = 0, 1, 2
NP_OF = {F32: np.float32, F16: np.float16, BF16: np.uint16}

_p = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int32
_f = C.c_float


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _build():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR, "oracle"], check=True)


def load_oracle() -> C.CDLL:
    if not os.path.exists(ORACLE_SO):
        _build()
    lib = C.CDLL(ORACLE_SO)
    lib.or_bf16_to_f16.restype = C.c_uint16
    lib.or_bf16_to_f16.argtypes = [C.c_uint16]
    lib.or_bf16_to_f16_vec.argtypes = [_p, _p, _i64]
    lib.or_f32_to_f16_rne.restype = C.c_uint16
    lib.or_f32_to_f16_rne.argtypes = [_f]
    lib.or_expf.restype = _f
    lib.or_expf.argtypes = [_f]
    lib.or_sincosf.argtypes = [_f, C.POINTER(_f), C.POINTER(_f)]
    lib.or_rope_inv_freq.argtypes = [_p, C.c_int, _f]
    lib.or_sumsq.restype = _f
    lib.or_sumsq.argtypes = [_p, C.c_int, C.c_int]
    lib.or_softmax_sum.restype = _f
    lib.or_softmax_sum.argtypes = [_p, C.c_int]
    lib.or_residual_rmsnorm.argtypes = [C.c_int, _p, _i64, _p, _i64, _p, _i64, _p, _i64,
                                        C.c_int, _f]
    lib.or_qk_norm_rope.argtypes = [C.c_int, _p, _p, _i64, _i64, C.c_int, C.c_int, C.c_int,
                                    C.c_int, C.c_int, C.c_int, _p, _p, _p, _i64, _f, _f]
    lib.or_silu_mul.argtypes = [C.c_int, _p, _i64, _p, _i64, _p, _i64, _i64, C.c_int]
    lib.or_embedding_gather.restype = _i64
    lib.or_embedding_gather.argtypes = [_p, C.c_int, _p, C.c_int, _p, _i64, C.c_int, C.c_int]
    lib.or_softmax_rows.argtypes = [_p, _i64, C.c_int, _i64]
    lib.or_sample_rows.argtypes = [_p, _i64, C.c_int, _i64, _p, _p, _i64, _p, _f, _f,
                                   C.c_int, _f, _p]
    lib.or_decode_attention.argtypes = [C.c_int, _p, _i64, _p, _i64, C.c_int, _p, _p, _i64,
                                        _p, _p, C.c_int, _i64, C.c_int, C.c_int, C.c_int]
    lib.or_kv_ring_advance.restype = C.c_int
    lib.or_apply_rope_interleaved.argtypes = [_p, _p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                              C.c_int, _f]
    lib.or_qk_norm_rope_kv.argtypes = [C.c_int, _p, _p, _p, _i64, _i64, _i64, C.c_int, C.c_int,
                                       C.c_int, C.c_int, C.c_int, C.c_int, _p, _p, _p, _p, _p,
                                       _i64, _p, _i64, _f, _f]
    lib.or_rmsnorm_gated.argtypes = [C.c_int, _p, _i64, _p, _i64, _p, _i64, _p, _i64, C.c_int, _f]
    lib.or_l2_normalize.argtypes = [C.c_int, _p, _i64, _i64, C.c_int, _f]
    lib.or_bf16_to_f32_weights.argtypes = [_p, _p, _i64, C.c_int]
    lib.or_f32_to_f16_trunc.restype = C.c_uint16
    lib.or_f32_to_f16_trunc.argtypes = [_f]
    lib.or_ane_pack.argtypes = [C.c_int, _p, _p, _i64, _i64, C.c_int, C.c_int]
    lib.or_ane_unpack.argtypes = [_p, _i64, _p, _i64, C.c_int, C.c_int]
    lib.or_kv_ring_advance.argtypes = [_p, _p, C.c_int]
    return lib


def load_ref():
    """The reference build, or None when it was not built (no reference tree)."""
    if not os.path.exists(REF_SO):
        return None
    lib = C.CDLL(REF_SO)
    lib.ref_bf16_to_f16_vec.argtypes = [_p, _p, _i64]
    lib.ref_rmsnorm.argtypes = [_p, _p, _p, C.c_int, _f]
    lib.ref_apply_rope_cached.argtypes = [_p, _p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.c_int, C.c_int, _f, _p, _p]
    lib.ref_rope_row.argtypes = [_p, _p, C.c_int, C.c_int, _f]
    lib.ref_silu_vec_inplace.argtypes = [_p, C.c_int]
    lib.ref_softmax.argtypes = [_p, C.c_int]
    lib.ref_rmsnorm_gated.argtypes = [_p, _p, _p, _p, C.c_int]
    lib.ref_l2_normalize.argtypes = [_p, C.c_int]
    lib.ref_load_weight.restype = C.c_int
    lib.ref_load_weight.argtypes = [C.c_char_p, C.c_char_p, _i64, C.c_int, _p]
    lib.ref_f32_to_f16_vec.argtypes = [_p, _p, _i64]
    lib.ref_f16_to_f32_vec.argtypes = [_p, _p, _i64]
    lib.ref_gqa_attention.argtypes = [_p, _p, _p, _p, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_int, C.c_int, C.c_int]
    lib.ref_sample_token.restype = C.c_int
    lib.ref_sample_token.argtypes = [_p, C.c_int, _f, _f, C.c_int, _f, _p, C.c_int, C.c_long,
                                     C.POINTER(_f)]
    lib.ref_sample_token_loop.argtypes = [_p, C.c_int, C.c_int, _f, _f, C.c_int, _f, _p, C.c_int,
                                          C.c_long, C.c_int, _p]
    lib.ref_write_ane_blobs.restype = C.c_int
    lib.ref_write_ane_blobs.argtypes = [C.c_char_p, C.c_char_p]
    lib.ref_layer_chain_f16.argtypes = [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64,
                                        C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _f, _f]
    return lib


class Oracle:
    """numpy-level wrappers over the C restatement."""

    def __init__(self):
        self.lib = load_oracle()

    def bf16_to_f16(self, a: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, dtype=np.uint16)
        out = np.empty_like(a)
        self.lib.or_bf16_to_f16_vec(_ptr(out), _ptr(a), a.size)
        return out

    def expf(self, x: np.ndarray) -> np.ndarray:
        f = self.lib.or_expf
        return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.float32)

    def sincosf(self, x):
        s, c = _f(), _f()
        self.lib.or_sincosf(float(x), C.byref(s), C.byref(c))
        return s.value, c.value

    def rope_inv_freq(self, rot_dim, theta):
        out = np.empty(rot_dim // 2, np.float32)
        self.lib.or_rope_inv_freq(_ptr(out), rot_dim, theta)
        return out

    def residual_rmsnorm(self, x, d, w, eps=1e-6):
        """Returns (x_after, y).  x, d: [rows, dim] of f32 / f16 / uint16(bf16)."""
        dt = dtype_code(x)
        x = np.ascontiguousarray(x).copy()
        rows, dim = x.shape
        y = np.empty_like(x)
        w = np.ascontiguousarray(w, np.float32)
        dd = None if d is None else np.ascontiguousarray(d, x.dtype)
        self.lib.or_residual_rmsnorm(dt, _ptr(x), dim, _ptr(dd), dim, _ptr(y), dim, _ptr(w),
                                     rows, dim, eps)
        return x, y

    def qk_norm_rope(self, qkv, nq, nkv, hd, qw, kw, pos, theta, eps=1e-6, rot_dim=None):
        """qkv: [rows, (nq + 2 nkv) * hd]; q and k normed + roped in place (copy returned)."""
        dt = dtype_code(qkv)
        qkv = np.ascontiguousarray(qkv).copy()
        rows, width = qkv.shape
        es = qkv.itemsize
        base = qkv.ctypes.data
        rot = hd if rot_dim is None else rot_dim
        self.lib.or_qk_norm_rope(dt, C.c_void_p(base), C.c_void_p(base + nq * hd * es),
                                 width, width, hd, hd, nq, nkv, hd, rot,
                                 _ptr(np.ascontiguousarray(qw, np.float32)),
                                 _ptr(np.ascontiguousarray(kw, np.float32)),
                                 _ptr(np.ascontiguousarray(pos, np.int32)), rows, theta, eps)
        return qkv

    def silu_mul(self, g, u):
        dt = dtype_code(g)
        g = np.ascontiguousarray(g)
        u = np.ascontiguousarray(u, g.dtype)
        rows, n = g.shape
        out = np.empty_like(g)
        self.lib.or_silu_mul(dt, _ptr(out), n, _ptr(g), n, _ptr(u), n, rows, n)
        return out

    def embedding_gather(self, table, ids, out_dtype=None):
        tdt = dtype_code(table)
        odt = tdt if out_dtype is None else out_dtype
        vocab, hidden = table.shape
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty((ids.size, hidden), NP_OF[odt])
        bad = self.lib.or_embedding_gather(_ptr(out), odt, _ptr(np.ascontiguousarray(table)), tdt,
                                           _ptr(ids), ids.size, vocab, hidden)
        return out, bad

    def softmax_rows(self, x):
        x = np.ascontiguousarray(x, np.float32).copy()
        rows, n = x.shape
        self.lib.or_softmax_rows(_ptr(x), rows, n, n)
        return x

    def sample_rows(self, logits, uniforms, history=None, history_len=None, temperature=0.6,
                    rep=1.2, ctx=256, freq=0.1):
        logits = np.ascontiguousarray(logits, np.float32)
        rows, vocab = logits.shape
        out = np.empty(rows, np.int32)
        if history is not None:
            history = np.ascontiguousarray(history, np.int32)
            hs = history.shape[1]
            if history_len is None:
                history_len = np.full(rows, hs, np.int32)
            history_len = np.ascontiguousarray(history_len, np.int32)
        else:
            hs = 0
        self.lib.or_sample_rows(_ptr(logits), rows, vocab, vocab, _ptr(history), _ptr(history_len),
                                hs, _ptr(np.ascontiguousarray(uniforms, np.float32)), temperature,
                                rep, ctx, freq, _ptr(out))
        return out

    def decode_attention(self, q, k_cache, v_cache, start, length):
        """q [B, H, hd]; caches [B, cap, Hk, hd]; start, length int32 [B]."""
        dt = dtype_code(q)
        q = np.ascontiguousarray(q)
        k_cache = np.ascontiguousarray(k_cache, q.dtype)
        v_cache = np.ascontiguousarray(v_cache, q.dtype)
        B, H, hd = q.shape
        _, cap, hk, _ = k_cache.shape
        out = np.empty_like(q)
        self.lib.or_decode_attention(dt, _ptr(out), H * hd, _ptr(q), H * hd, hd, _ptr(k_cache),
                                     _ptr(v_cache), cap * hk * hd,
                                     _ptr(np.ascontiguousarray(start, np.int32)),
                                     _ptr(np.ascontiguousarray(length, np.int32)), cap, B, H, hk,
                                     hd)
        return out

    def apply_rope_interleaved(self, q, k, rot_dim, pos, theta):
        """apply_rope_cached without tables (the reference's fallback) on
        fp32 q [n_q, hd] and k [n_kv, hd]; returns new arrays."""
        q, k = np.array(q, np.float32, copy=True), np.array(k, np.float32, copy=True)
        self.lib.or_apply_rope_interleaved(_ptr(q), _ptr(k), q.shape[0], k.shape[0], q.shape[1],
                                           k.shape[1], rot_dim, pos, theta)
        return q, k

    def qk_norm_rope_kv(self, qkv, nq, nkv, hd, qw, kw, pos, theta, k_cache, v_cache, slots,
                        per_row_cache=False, eps=1e-6):
        """qkv [rows, (nq + 2 nkv) hd]; caches [cap, nkv, hd] shared by all rows, or
        [rows, cap, nkv, hd] with per_row_cache.  Returns (qkv, k_cache, v_cache) copies."""
        dt = dtype_code(qkv)
        qkv = np.ascontiguousarray(qkv).copy()
        kc = np.ascontiguousarray(k_cache).copy()
        vc = np.ascontiguousarray(v_cache).copy()
        rows, width = qkv.shape
        es = qkv.itemsize
        base = qkv.ctypes.data
        crs = (kc.size // rows) if per_row_cache else 0
        self.lib.or_qk_norm_rope_kv(dt, C.c_void_p(base), C.c_void_p(base + nq * hd * es),
                                    C.c_void_p(base + (nq + nkv) * hd * es), width, width, width,
                                    hd, hd, hd, nq, nkv, hd,
                                    _ptr(np.ascontiguousarray(qw, np.float32)),
                                    _ptr(np.ascontiguousarray(kw, np.float32)),
                                    _ptr(np.ascontiguousarray(pos, np.int32)), _ptr(kc), _ptr(vc), crs,
                                    _ptr(np.ascontiguousarray(slots, np.int32)), rows, theta, eps)
        return qkv, kc, vc

    def rmsnorm_gated(self, x, z, w, eps=1e-6):
        dt = dtype_code(x)
        x = np.ascontiguousarray(x)
        z = np.ascontiguousarray(z, x.dtype)
        rows, dim = x.shape
        out = np.empty_like(x)
        self.lib.or_rmsnorm_gated(dt, _ptr(out), dim, _ptr(x), dim, _ptr(z), dim,
                                  _ptr(np.ascontiguousarray(w, np.float32)), rows, dim, eps)
        return out

    def l2_normalize(self, x, scale=1.0):
        dt = dtype_code(x)
        x = np.ascontiguousarray(x).copy()
        rows, dim = x.shape
        self.lib.or_l2_normalize(dt, _ptr(x), dim, rows, dim, scale)
        return x

    def bf16_to_f32_weights(self, b, add_one):
        b = np.ascontiguousarray(b, np.uint16)
        out = np.empty(b.shape, np.float32)
        self.lib.or_bf16_to_f32_weights(_ptr(out), _ptr(b), b.size, int(add_one))
        return out

    def ane_pack(self, x, round_mode=0, spatial=32, surface=None):
        """x [tokens, channels] f32 -> surfaces [ceil(tokens/spatial), channels, spatial]
        uint16 (fp16 bits); slots without a token keep `surface`'s values (zeros)."""
        x = np.ascontiguousarray(x, np.float32)
        t, c = x.shape
        nsurf = (t + spatial - 1) // spatial
        if surface is None:
            surface = np.zeros((nsurf, c, spatial), np.uint16)
        surface = np.ascontiguousarray(surface, np.uint16).copy()
        self.lib.or_ane_pack(round_mode, _ptr(surface), _ptr(x), c, t, c, spatial)
        return surface

    def ane_unpack(self, surface, tokens, spatial=32):
        surface = np.ascontiguousarray(surface, np.uint16)
        c = surface.shape[1]
        out = np.empty((tokens, c), np.float32)
        self.lib.or_ane_unpack(_ptr(out), c, _ptr(surface), tokens, c, spatial)
        return out

    def kv_ring_advance(self, start, length, capacity):
        s, n = C.c_int32(start), C.c_int32(length)
        slot = self.lib.or_kv_ring_advance(C.byref(s), C.byref(n), capacity)
        return slot, s.value, n.value


def dtype_code(a: np.ndarray) -> int:
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.float16:
        return F16
    if a.dtype == np.uint16:
        return BF16
    raise TypeError(a.dtype)


def f16_ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in fp16 units in the last place between two fp16 arrays
    (ordered-integer distance; +0 and -0 are 0 apart)."""
    ai = a.view(np.int16).astype(np.int32)
    bi = b.view(np.int16).astype(np.int32)
    ai = np.where(ai < 0, -(ai & 0x7FFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFF), bi)
    return np.abs(ai - bi)


def f32_ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)
