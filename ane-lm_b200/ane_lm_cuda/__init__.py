"""Python access to libane_cuda.so, the sm_100a backend of ANE-LM's layer-op,
sampler and BF16->FP16 convert path.

``lib()`` returns the ctypes handle of the C ABI (include/ane_cuda.h).  The
wrappers below take torch CUDA tensors, check shapes / dtypes / devices and
pass raw device pointers and torch's current stream.  There is no fallback:
if the shared library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libane_cuda.so")
HEADER = os.path.join(REPO, "include", "ane_cuda.h")

OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
F32, F16, BF16 = 0, 1, 2
FLAG_BAD_TOKEN_ID = 0x1
ROUND_NEAREST, ROUND_TRUNCATE = 0, 1
FLAG_BAD_CACHE = 0x2
FLAG_WAIT_TIMEOUT = 0x4

_p = C.c_void_p
_i64 = C.c_int64
_i = C.c_int
_f = C.c_float

_SIGS = {
    "ane_cuda_abi_version": (_i, []),
    "ane_cuda_status_string": (C.c_char_p, [_i]),
    "ane_cuda_last_error": (C.c_char_p, []),
    "ane_cuda_read_status_flags": (_i, [C.POINTER(C.c_uint32), _i]),
    "ane_cuda_bf16_to_f16": (_i, [_p, _p, _i64, _p]),
    "ane_cuda_embedding_gather": (_i, [_p, _i, _p, _i, _p, _i64, _i, _i, _p]),
    "ane_cuda_embedding_rmsnorm": (_i, [_i, _p, _i64, _p, _i64, _p, _i, _p, _i64, _i, _i, _i, _p,
                                        _f, _p]),
    "ane_cuda_residual_rmsnorm": (_i, [_i, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _f, _p]),
    "ane_cuda_qk_norm_rope": (_i, [_i, _p, _p, _i64, _i64, _i, _i, _i, _i, _i, _i, _p, _p, _p,
                                   _i64, _f, _f, _p]),
    "ane_cuda_apply_rope_cached": (_i, [_p, _p, _i, _i, _i, _i, _i, _i, _i, _f, _p, _p, _p]),
    "ane_cuda_silu_mul": (_i, [_i, _p, _i64, _p, _i64, _p, _i64, _i64, _i, _p]),
    "ane_cuda_silu_inplace": (_i, [_i, _p, _i64, _p]),
    "ane_cuda_mul_sigmoid_inplace": (_i, [_i, _p, _p, _i64, _p]),
    "ane_cuda_softmax_rows": (_i, [_p, _i64, _i, _i64, _p]),
    "ane_cuda_sample_rows": (_i, [_p, _i64, _i, _i64, _p, _p, _i64, _p, _f, _f, _i, _f, _p, _p]),
    "ane_cuda_write_ane_blobs": (_i, [C.c_char_p, C.c_char_p, C.POINTER(_i64), _p]),
    "ane_cuda_convert_model": (_i, [C.c_char_p, C.c_char_p, C.POINTER(_i64), _p]),
    "ane_cuda_qk_norm_rope_kv": (_i, [_i, _p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _i,
                                      _p, _p, _p, _p, _p, _i64, _p, _i, _i64, _f, _f, _p]),
    "ane_cuda_rmsnorm_gated": (_i, [_i, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i, _f, _p]),
    "ane_cuda_l2_normalize": (_i, [_i, _p, _i64, _i64, _i, _f, _p]),
    "ane_cuda_bf16_to_f32": (_i, [_p, _p, _i64, _i, _p]),
    "ane_cuda_ane_pack": (_i, [_i, _p, _p, _i64, _i64, _i, _i, _p]),
    "ane_cuda_ane_unpack": (_i, [_p, _i64, _p, _i64, _i, _i, _p]),
    "ane_cuda_decode_attention_workspace_size": (_i64, [_i64, _i, _i, _i, _i]),
    "ane_cuda_decode_attention_static_capacity": (_i64, []),
    "ane_cuda_decode_attention_static": (_i, [_i, _p, _i64, _p, _i64, _i, _p, _p, _i64, _p, _p,
                                              _i, _i64, _i, _i, _i, _i, _p]),
    "ane_cuda_decode_attention": (_i, [_i, _p, _i64, _p, _i64, _i, _p, _p, _i64, _p, _p, _i,
                                       _i64, _i, _i, _i, _i, _p, _i64, _p]),
}

_lib = None


class AneCudaError(RuntimeError):
    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn}: status {status}: {msg}")
        self.status = status


def lib() -> C.CDLL:
    """The loaded C ABI.  Raises if libane_cuda.so has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` "
                              "(or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def declared_symbols() -> list[str]:
    """Every ane_cuda_* function declared in include/ane_cuda.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"ANE_CUDA_API\s+[\w\s\*]*?\b(ane_cuda_\w+)\s*\(", text)))


def _check(fn: str, st: int):
    if st != OK:
        raise AneCudaError(fn, st, lib().ane_cuda_last_error().decode())


# --------------------------------------------------------------------------
# torch-tensor wrappers
# --------------------------------------------------------------------------
def _torch():
    import torch
    return torch


def _dt(t) -> int:
    torch = _torch()
    m = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
    if t.dtype not in m:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return m[t.dtype]


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(t):
    torch = _torch()
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("tensors must be on a CUDA device")


def read_status_flags(clear: bool = True) -> int:
    v = C.c_uint32(0)
    _check("read_status_flags", lib().ane_cuda_read_status_flags(C.byref(v), int(clear)))
    return v.value


def bf16_to_f16(inp, out=None):
    """inp: int16/uint16/bfloat16 tensor of BF16 bits -> int16 tensor of FP16 bits."""
    torch = _torch()
    _cuda(inp)
    inp = inp.contiguous()
    if out is None:
        out = torch.empty(inp.shape, dtype=torch.int16, device=inp.device)
    _check("bf16_to_f16", lib().ane_cuda_bf16_to_f16(_ptr(out), _ptr(inp), inp.numel(), _stream(inp)))
    return out


def embedding_gather(table, ids, out_dtype=None, out=None):
    torch = _torch()
    _cuda(table, ids)
    vocab, hidden = table.shape
    odt = table.dtype if out_dtype is None else out_dtype
    if out is None:
        out = torch.empty((ids.numel(), hidden), dtype=odt, device=table.device)
    ids = ids.to(torch.int32).contiguous()
    _check("embedding_gather", lib().ane_cuda_embedding_gather(
        _ptr(out), _dt(out), _ptr(table), _dt(table), _ptr(ids), ids.numel(), vocab, hidden,
        _stream(table)))
    return out


def embedding_rmsnorm(table, ids, weight, x=None, accumulate=False, out_dtype=None, out=None,
                      eps=1e-6):
    """x = table[ids] widened to out_dtype (or x += table[ids] with accumulate);
    returns rmsnorm(x) * weight.  x is written in place when given."""
    torch = _torch()
    _cuda(table, ids, weight, x, out)
    vocab, hidden = table.shape
    odt = (table.dtype if out_dtype is None else out_dtype) if x is None else x.dtype
    ids = ids.to(torch.int32).contiguous()
    if x is None:
        x = torch.empty((ids.numel(), hidden), dtype=odt, device=table.device)
    if out is None:
        out = torch.empty_like(x)
    _check("embedding_rmsnorm", lib().ane_cuda_embedding_rmsnorm(
        _dt(x), _ptr(x), x.stride(0), _ptr(out), out.stride(0), _ptr(table), _dt(table), _ptr(ids),
        ids.numel(), vocab, hidden, int(accumulate), _ptr(weight), eps, _stream(table)))
    return x, out


def residual_rmsnorm(x, d, weight, out=None, eps=1e-6):
    """x += d (in place, when d is given); returns rmsnorm(x) * weight."""
    torch = _torch()
    _cuda(x, d, weight)
    rows, dim = x.shape
    if out is None:
        out = torch.empty_like(x)
    _check("residual_rmsnorm", lib().ane_cuda_residual_rmsnorm(
        _dt(x), _ptr(x), x.stride(0), _ptr(d), 0 if d is None else d.stride(0), _ptr(out),
        out.stride(0), _ptr(weight), rows, dim, eps, _stream(x)))
    return out


def qk_norm_rope(qkv, q_weight, k_weight, positions, n_q_heads, n_kv_heads, head_dim,
                 theta=1e6, eps=1e-6, rot_dim=None):
    """In place on the q and k heads of qkv [rows, (n_q + 2 n_kv) * head_dim]."""
    _cuda(qkv, q_weight, k_weight, positions)
    rows, width = qkv.shape
    es = qkv.element_size()
    k = C.c_void_p(qkv.data_ptr() + n_q_heads * head_dim * es)
    rot = head_dim if rot_dim is None else rot_dim
    _check("qk_norm_rope", lib().ane_cuda_qk_norm_rope(
        _dt(qkv), _ptr(qkv), k, qkv.stride(0), qkv.stride(0), head_dim, head_dim, n_q_heads,
        n_kv_heads, head_dim, rot, _ptr(q_weight), _ptr(k_weight), _ptr(positions), rows, theta,
        eps, _stream(qkv)))
    return qkv


def silu_mul(gate, up, out=None):
    torch = _torch()
    _cuda(gate, up)
    rows, n = gate.shape
    if out is None:
        out = torch.empty_like(gate)
    _check("silu_mul", lib().ane_cuda_silu_mul(
        _dt(gate), _ptr(out), out.stride(0), _ptr(gate), gate.stride(0), _ptr(up), up.stride(0),
        rows, n, _stream(gate)))
    return out


def softmax_rows(x):
    _cuda(x)
    rows, n = x.shape
    _check("softmax_rows", lib().ane_cuda_softmax_rows(_ptr(x), rows, n, x.stride(0), _stream(x)))
    return x


def write_ane_blobs(safetensors_path: str, output_dir: str) -> int:
    """`ane-lm convert` of one .safetensors file; returns the number of blobs."""
    n = _i64(0)
    _check("write_ane_blobs", lib().ane_cuda_write_ane_blobs(
        safetensors_path.encode(), output_dir.encode(), C.byref(n), None))
    return n.value


def convert_model(model_dir: str, output_dir: str) -> int:
    """`ane-lm convert` of a model directory (all shards); returns the blob count."""
    n = _i64(0)
    _check("convert_model", lib().ane_cuda_convert_model(
        model_dir.encode(), output_dir.encode(), C.byref(n), None))
    return n.value


def sample_rows(logits, uniforms, history=None, history_len=None, temperature=0.6,
                repetition_penalty=1.2, repetition_context=256, frequency_penalty=0.1, out=None):
    torch = _torch()
    _cuda(logits, uniforms, history, history_len)
    rows, vocab = logits.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    hs = 0 if history is None else history.stride(0)
    _check("sample_rows", lib().ane_cuda_sample_rows(
        _ptr(logits), rows, vocab, logits.stride(0), _ptr(history), _ptr(history_len), hs,
        _ptr(uniforms), temperature, repetition_penalty, repetition_context, frequency_penalty,
        _ptr(out), _stream(logits)))
    return out


def decode_attention_workspace_size(batch, n_heads, n_kv_heads, head_dim, max_len) -> int:
    return int(lib().ane_cuda_decode_attention_workspace_size(batch, n_heads, n_kv_heads,
                                                              head_dim, max_len))


def decode_attention(q, k_cache, v_cache, cache_start, cache_len, max_len=None, out=None,
                     workspace=None):
    """q [batch, n_heads, head_dim]; k_cache, v_cache [batch, capacity, n_kv, head_dim];
    cache_start, cache_len int32 [batch].  Returns out [batch, n_heads, head_dim].
    workspace: a uint8 tensor of decode_attention_workspace_size() bytes (any
    contents; only the call in flight uses it), or None for the library-held one."""
    torch = _torch()
    _cuda(q, k_cache, v_cache, cache_start, cache_len, workspace)
    batch, n_heads, head_dim = q.shape
    _, capacity, n_kv, hd2 = k_cache.shape
    if hd2 != head_dim or v_cache.shape != k_cache.shape:
        raise ValueError("q / cache shapes disagree")
    if max_len is None:
        max_len = capacity
    if out is None:
        out = torch.empty_like(q)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check("decode_attention", lib().ane_cuda_decode_attention(
        _dt(q), _ptr(out), out.stride(0), _ptr(q), q.stride(0), q.stride(1), _ptr(k_cache),
        _ptr(v_cache), k_cache.stride(0), _ptr(cache_start), _ptr(cache_len), capacity, batch,
        n_heads, n_kv, head_dim, max_len, _ptr(workspace), ws_bytes, _stream(q)))
    return out


def decode_attention_static(q, k_cache, v_cache, cache_start, cache_len, max_len=None, out=None):
    """decode_attention with the split scratch in a fixed device array: allocates
    nothing; calls must not overlap in time (order them on one stream)."""
    torch = _torch()
    _cuda(q, k_cache, v_cache, cache_start, cache_len)
    batch, n_heads, head_dim = q.shape
    _, capacity, n_kv, _ = k_cache.shape
    if max_len is None:
        max_len = capacity
    if out is None:
        out = torch.empty_like(q)
    _check("decode_attention_static", lib().ane_cuda_decode_attention_static(
        _dt(q), _ptr(out), out.stride(0), _ptr(q), q.stride(0), q.stride(1), _ptr(k_cache),
        _ptr(v_cache), k_cache.stride(0), _ptr(cache_start), _ptr(cache_len), capacity, batch,
        n_heads, n_kv, head_dim, max_len, _stream(q)))
    return out


def ane_pack(x, round_mode=ROUND_NEAREST, spatial=32, surface=None):
    """x [tokens, channels] float32 -> surfaces [ceil(tokens/spatial), channels, spatial]
    int16 (fp16 bits).  Slots without a token keep `surface`'s contents (zeros)."""
    torch = _torch()
    _cuda(x, surface)
    tokens, channels = x.shape
    if surface is None:
        surface = torch.zeros(((tokens + spatial - 1) // spatial, channels, spatial),
                              dtype=torch.int16, device=x.device)
    _check("ane_pack", lib().ane_cuda_ane_pack(round_mode, _ptr(surface), _ptr(x), x.stride(0),
                                               tokens, channels, spatial, _stream(x)))
    return surface


def ane_unpack(surface, tokens, spatial=32, out=None):
    """surfaces [n, channels, spatial] of fp16 bits -> out [tokens, channels] float32."""
    torch = _torch()
    _cuda(surface, out)
    channels = surface.shape[1]
    if out is None:
        out = torch.empty((tokens, channels), dtype=torch.float32, device=surface.device)
    _check("ane_unpack", lib().ane_cuda_ane_unpack(_ptr(out), out.stride(0), _ptr(surface), tokens,
                                                   channels, spatial, _stream(surface)))
    return out


def rmsnorm_gated(x, z, weight, out=None, eps=1e-6):
    """((rmsnorm(x) * weight) / (1 + exp(-z))) * z over rows of x [rows, dim]."""
    torch = _torch()
    _cuda(x, z, weight)
    rows, dim = x.shape
    if out is None:
        out = torch.empty_like(x)
    _check("rmsnorm_gated", lib().ane_cuda_rmsnorm_gated(
        _dt(x), _ptr(out), out.stride(0), _ptr(x), x.stride(0), _ptr(z), z.stride(0), _ptr(weight),
        rows, dim, eps, _stream(x)))
    return out


def l2_normalize(x, scale=1.0):
    """In place over rows of x [rows, dim]: x / sqrt(sum(x^2) + 1e-12) * scale."""
    _cuda(x)
    rows, dim = x.shape
    _check("l2_normalize", lib().ane_cuda_l2_normalize(_dt(x), _ptr(x), x.stride(0), rows, dim,
                                                       scale, _stream(x)))
    return x


def bf16_to_f32(bits, add_one=False, out=None):
    """BF16 bits (int16 / uint16 / bfloat16 tensor) -> float32, optionally + 1."""
    torch = _torch()
    _cuda(bits)
    bits = bits.contiguous()
    if out is None:
        out = torch.empty(bits.shape, dtype=torch.float32, device=bits.device)
    _check("bf16_to_f32", lib().ane_cuda_bf16_to_f32(_ptr(out), _ptr(bits), bits.numel(),
                                                     int(add_one), _stream(bits)))
    return out


def qk_norm_rope_kv(qkv, q_weight, k_weight, positions, n_q_heads, n_kv_heads, head_dim,
                    k_cache, v_cache, slots, theta=1e6, eps=1e-6):
    """qk_norm_rope on qkv [rows, (n_q + 2 n_kv) * head_dim] in place, and row r's k heads
    (after RoPE) and v heads written to ring slot slots[r] of k_cache / v_cache:
    [cap, n_kv, head_dim] shared by all rows, or [rows, cap, n_kv, head_dim] per row."""
    _cuda(qkv, q_weight, k_weight, positions, k_cache, v_cache, slots)
    rows, width = qkv.shape
    es = qkv.element_size()
    base = qkv.data_ptr()
    k = C.c_void_p(base + n_q_heads * head_dim * es)
    v = C.c_void_p(base + (n_q_heads + n_kv_heads) * head_dim * es)
    crs = k_cache.stride(0) if k_cache.dim() == 4 else 0
    capacity = k_cache.shape[-3]
    _check("qk_norm_rope_kv", lib().ane_cuda_qk_norm_rope_kv(
        _dt(qkv), _ptr(qkv), k, v, qkv.stride(0), qkv.stride(0), qkv.stride(0), head_dim, head_dim,
        head_dim, n_q_heads, n_kv_heads, head_dim, _ptr(q_weight), _ptr(k_weight), _ptr(positions),
        _ptr(k_cache), _ptr(v_cache), crs, _ptr(slots), capacity, rows, theta, eps, _stream(qkv)))
    return qkv
