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
