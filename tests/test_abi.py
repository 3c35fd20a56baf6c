"""The C-ABI library loads and exports every symbol include/styx_moe.h
declares (no GPU needed, no compute calls)."""
import ctypes as C
import os

import pytest

from styx_b200 import _lib


@pytest.fixture(scope="module")
def libso():
    from styx_b200 import build
    build.build()
    return C.CDLL(_lib.LIB_PATH)


def test_header_declares_the_hot_path():
    names = _lib.header_functions()
    for need in ("styx_init", "styx_topk_softmax", "styx_mul_mat_vec_id", "styx_swiglu",
                 "styx_moe_reduce", "styx_gather_slabs", "styx_moe_block"):
        assert need in names


def test_every_declared_symbol_is_exported(libso):
    missing = [n for n in _lib.header_functions() if not hasattr(libso, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert set(_lib.header_functions()) <= set(_lib._SIGS)


def test_built_for_sm100a_only():
    """The build passes only sm_100a to nvcc (no multi-arch dispatch)."""
    from styx_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_errors_without_gpu_are_loud(libso):
    """With no GPU, styx_init fails with a message (no CPU fallback)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    L = _lib.lib()
    h = C.c_void_p()
    rc = L.styx_init(0, C.byref(h))
    assert rc != 0
    assert L.styx_last_error()


def test_workspace_bytes_and_dims_validation(libso):
    L = _lib.lib()
    d = _lib.MoeDims(2048, 768, 128, 8, 1, 1e-6)
    n = C.c_uint64()
    assert L.styx_moe_workspace_bytes(C.byref(d), C.byref(n)) == 0
    assert n.value >= 4 * (2048 + 128 + 8 * 768)
    bad = _lib.MoeDims(2000, 768, 128, 8, 1, 1e-6)
    assert L.styx_moe_workspace_bytes(C.byref(bad), C.byref(n)) == _lib.STYX_EINVAL
    assert b"n_embd" in L.styx_last_error()
    bad = _lib.MoeDims(2048, 768, 128, 17, 1, 1e-6)
    assert L.styx_moe_workspace_bytes(C.byref(bad), C.byref(n)) == _lib.STYX_EINVAL


def test_library_has_no_oracle_dependency(libso):
    """The product library never links the oracle."""
    import subprocess
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in out
    with open(_lib.LIB_PATH, "rb") as f:
        blob = f.read()
    assert b"or_moe_block" not in blob and b"liboracle" not in blob
    assert os.path.getsize(_lib.LIB_PATH) > 0
