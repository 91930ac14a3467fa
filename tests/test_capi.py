"""CPU checks of the C ABI library: it loads without a GPU, exports every
symbol include/ane_cuda.h declares, and rejects bad arguments on the host
before touching CUDA."""
import ctypes as C
import os
import subprocess

import pytest

import ane_lm_cuda as A


def test_library_exports_every_declared_symbol(ane):
    declared = A.declared_symbols()
    assert len(declared) >= 14
    out = subprocess.run(["nm", "-D", "--defined-only", A.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(ane.lib(), s)
    # nothing but the ABI is exported
    assert all(s.startswith("ane_cuda_") or s.startswith("_ZN6ane_lm4cuda") or s in ("_init", "_fini")
               for s in exported), sorted(exported)[:20]


def test_abi_version_and_status_strings(ane):
    L = ane.lib()
    assert L.ane_cuda_abi_version() == 1
    assert L.ane_cuda_status_string(0) == b"ok"
    assert L.ane_cuda_status_string(1) == b"invalid argument"
    assert L.ane_cuda_status_string(99) == b"unknown status"


def _p(v):
    return C.c_void_p(v)


@pytest.mark.parametrize("call", [
    lambda L: L.ane_cuda_bf16_to_f16(_p(16), _p(32), -1, None),
    lambda L: L.ane_cuda_bf16_to_f16(None, _p(32), 8, None),
    lambda L: L.ane_cuda_embedding_gather(_p(16), 0, _p(16), 0, _p(16), 4, 0, 8, None),
    lambda L: L.ane_cuda_embedding_gather(_p(16), 7, _p(16), 0, _p(16), 4, 10, 8, None),
    lambda L: L.ane_cuda_residual_rmsnorm(0, _p(16), 8, None, 0, _p(16), 8, None, 2, 8, 1e-6, None),
    lambda L: L.ane_cuda_residual_rmsnorm(5, _p(16), 8, None, 0, _p(16), 8, _p(16), 2, 8, 1e-6, None),
    lambda L: L.ane_cuda_residual_rmsnorm(1, _p(16), 4, None, 0, _p(16), 8, _p(16), 2, 8, 1e-6, None),
    lambda L: L.ane_cuda_qk_norm_rope(1, _p(16), _p(16), 8, 8, 2, 2, 1, 1, 2, 3, None, None,
                                      _p(16), 1, 1e6, 1e-6, None),
    lambda L: L.ane_cuda_qk_norm_rope(1, _p(16), _p(16), 8, 8, 2, 2, 1, 1, 2, 2, _p(16), None,
                                      _p(16), 1, 1e6, 1e-6, None),
    lambda L: L.ane_cuda_qk_norm_rope(1, _p(16), _p(16), 8, 8, 2, 2, 1, 1, 2, 2, None, None,
                                      None, 1, 1e6, 1e-6, None),
    lambda L: L.ane_cuda_silu_mul(1, _p(16), 4, _p(16), 8, _p(16), 8, 2, 8, None),
    lambda L: L.ane_cuda_silu_inplace(1, None, 8, None),
    lambda L: L.ane_cuda_mul_sigmoid_inplace(1, _p(16), None, 8, None),
    lambda L: L.ane_cuda_softmax_rows(_p(16), 2, 8, 4, None),
    lambda L: L.ane_cuda_sample_rows(_p(16), 2, 8, 4, None, None, 0, _p(16), 0.6, 1.2, 256, 0.1,
                                     _p(16), None),
    lambda L: L.ane_cuda_sample_rows(_p(16), 2, 8, 8, _p(16), None, 4, _p(16), 0.6, 1.2, 256,
                                     0.1, _p(16), None),
    lambda L: L.ane_cuda_read_status_flags(None, 0),
    # decode attention: bad dtype, heads not a multiple of kv heads, null
    # pointer, output stride below the heads, negative max_len
    lambda L: L.ane_cuda_decode_attention(7, _p(16), 2048, _p(16), 2048, 128, _p(16), _p(16),
                                          1 << 20, _p(16), _p(16), 1024, 1, 16, 8, 128, 64, None,
                                          0, None),
    lambda L: L.ane_cuda_decode_attention(0, _p(16), 2048, _p(16), 2048, 128, _p(16), _p(16),
                                          1 << 20, _p(16), _p(16), 1024, 1, 12, 8, 128, 64, None,
                                          0, None),
    lambda L: L.ane_cuda_decode_attention(0, None, 2048, _p(16), 2048, 128, _p(16), _p(16),
                                          1 << 20, _p(16), _p(16), 1024, 1, 16, 8, 128, 64, None,
                                          0, None),
    lambda L: L.ane_cuda_decode_attention(0, _p(16), 100, _p(16), 2048, 128, _p(16), _p(16),
                                          1 << 20, _p(16), _p(16), 1024, 1, 16, 8, 128, 64, None,
                                          0, None),
    lambda L: L.ane_cuda_decode_attention(0, _p(16), 2048, _p(16), 2048, 128, _p(16), _p(16),
                                          1 << 20, _p(16), _p(16), 1024, 1, 16, 8, 128, -1, None,
                                          0, None),
    # a caller workspace that is too small
    lambda L: L.ane_cuda_decode_attention(0, _p(16), 2048, _p(16), 2048, 128, _p(16), _p(16),
                                          1 << 20, _p(16), _p(16), 1024, 1, 16, 8, 128, 1024,
                                          _p(256), 16, None),
    # the allocation-free form: more split scratch than its fixed array
    lambda L: L.ane_cuda_decode_attention_static(0, _p(16), 4096, _p(16), 4096, 128, _p(16),
                                                 _p(16), 1 << 22, _p(16), _p(16), 8192, 64, 32, 8,
                                                 128, 8192, None),
    lambda L: L.ane_cuda_qk_norm_rope_kv(1, _p(16), _p(16), None, 512, 512, 512, 128, 128, 128, 2,
                                         1, 128, _p(16), _p(16), _p(16), _p(16), _p(16), 0, _p(16),
                                         64, 1, 1e6, 1e-6, None),
    lambda L: L.ane_cuda_qk_norm_rope_kv(1, _p(16), _p(16), _p(16), 512, 512, 512, 128, 128, 128, 2,
                                         1, 128, _p(16), _p(16), _p(16), _p(16), _p(16), 0, _p(16),
                                         0, 1, 1e6, 1e-6, None),
    lambda L: L.ane_cuda_rmsnorm_gated(0, _p(16), 128, _p(16), 64, _p(16), 128, _p(16), 2, 128,
                                       1e-6, None),
    lambda L: L.ane_cuda_rmsnorm_gated(0, _p(16), 128, _p(16), 128, None, 128, _p(16), 2, 128,
                                       1e-6, None),
    lambda L: L.ane_cuda_l2_normalize(0, None, 128, 2, 128, 1.0, None),
    lambda L: L.ane_cuda_l2_normalize(9, _p(16), 128, 2, 128, 1.0, None),
    lambda L: L.ane_cuda_bf16_to_f32(_p(16), _p(16), -1, 1, None),
    lambda L: L.ane_cuda_ane_pack(2, _p(16), _p(16), 8, 4, 8, 32, None),
    lambda L: L.ane_cuda_ane_pack(0, _p(16), _p(16), 8, 4, 8, 0, None),
    lambda L: L.ane_cuda_ane_unpack(_p(16), 4, _p(16), 4, 8, 32, None),
])
def test_invalid_arguments_rejected_on_host(ane, call):
    L = ane.lib()
    assert call(L) == A.ERR_INVALID_ARG
    assert L.ane_cuda_last_error() != b""


def test_zero_sized_calls_are_no_ops(ane):
    L = ane.lib()
    assert L.ane_cuda_bf16_to_f16(None, None, 0, None) == A.OK
    assert L.ane_cuda_residual_rmsnorm(1, None, 8, None, 0, None, 8, None, 0, 8, 1e-6, None) == A.OK
    assert L.ane_cuda_silu_mul(1, None, 8, None, 8, None, 8, 0, 8, None) == A.OK
    assert L.ane_cuda_sample_rows(None, 0, 8, 8, None, None, 0, None, 0.6, 1.2, 256, 0.1, None,
                                  None) == A.OK


def test_zero_sized_calls_of_the_next_rows(ane):
    L = ane.lib()
    assert L.ane_cuda_decode_attention(0, _p(16), 2048, _p(16), 2048, 128, _p(16), _p(16), 1 << 20,
                                       _p(16), _p(16), 1024, 0, 16, 8, 128, 1024, None, 0,
                                       None) == A.OK
    assert L.ane_cuda_ane_pack(0, None, None, 8, 0, 8, 32, None) == A.OK
    assert L.ane_cuda_ane_unpack(None, 8, None, 0, 8, 32, None) == A.OK
    assert L.ane_cuda_rmsnorm_gated(0, None, 8, None, 8, None, 8, None, 0, 8, 1e-6, None) == A.OK
    assert L.ane_cuda_l2_normalize(0, None, 8, 0, 8, 1.0, None) == A.OK
    assert L.ane_cuda_bf16_to_f32(None, None, 0, 0, None) == A.OK


@pytest.mark.parametrize("head_dim,heads,kv", [(96, 16, 8), (128, 32, 2)])
def test_decode_attention_unsupported_shapes(ane, head_dim, heads, kv):
    """head_dim other than 64/128/256, or more than 8 q heads per kv head."""
    L = ane.lib()
    st = L.ane_cuda_decode_attention(0, _p(16), heads * head_dim, _p(16), heads * head_dim,
                                     head_dim, _p(16), _p(16), 1 << 22, _p(16), _p(16), 1024, 1,
                                     heads, kv, head_dim, 64, None, 0, None)
    assert st == A.ERR_UNSUPPORTED


def test_workspace_size_rule(ane):
    """No workspace with one split (max_len <= 64); (m, l) + o per split
    otherwise, each 256-byte aligned."""
    L = ane.lib()
    assert L.ane_cuda_decode_attention_workspace_size(4, 16, 8, 128, 64) == 0
    n = L.ane_cuda_decode_attention_workspace_size(4, 16, 8, 128, 4096)
    splits = 4096 // 64
    r = lambda v: (v + 255) // 256 * 256  # noqa: E731
    assert n == r(4 * 16 * splits * 2 * 4) + r(4 * 16 * splits * 128 * 4)
    assert L.ane_cuda_decode_attention_workspace_size(-1, 16, 8, 128, 64) == -1
    assert L.ane_cuda_decode_attention_static_capacity() == 16 << 20


def test_unsupported_window_is_reported(ane):
    L = ane.lib()
    st = L.ane_cuda_sample_rows(_p(16), 1, 8, 8, _p(16), _p(16), 100000, _p(16), 0.6, 1.2, 100000,
                                0.1, _p(16), None)
    assert st == A.ERR_UNSUPPORTED
    assert b"window" in L.ane_cuda_last_error()


def test_product_path_has_no_oracle_dependency():
    """The shipped library links no oracle code and the package imports none."""
    pkg = os.path.dirname(A.LIB_PATH)
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                text = open(os.path.join(root, f)).read()
                assert "oracle" not in text.lower(), f
    out = subprocess.run(["nm", "-D", A.LIB_PATH], capture_output=True, text=True).stdout
    assert "or_" + "expf" not in out and "ref_" + "rmsnorm" not in out
