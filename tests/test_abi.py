"""CPU checks of the C-ABI library: it loads, exports exactly what include/rtd.h
declares, and its host-only entry points behave without a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from runtimed_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADER = os.path.join(ROOT, "include", "rtd.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rtd_[a-z0-9_]+)\s*\(", text)))


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    return sorted({line.split()[-1] for line in out.splitlines() if " T " in line and "rtd_" in line})


def test_library_loads_and_binds_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_exports_are_exactly_the_header():
    assert exported_symbols() == declared_symbols()


def test_block_geometry_matches_reference_table():
    # crates/runtimed-gguf/src/quant/dtype.rs:49-64
    L = _lib.lib()
    e, b = ctypes.c_int64(), ctypes.c_int64()
    table = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 6: (32, 22), 8: (32, 34), 10: (256, 84),
             11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
    for t, want in table.items():
        assert L.rtd_block_geometry(t, ctypes.byref(e), ctypes.byref(b)) == 0
        assert (e.value, b.value) == want
    assert L.rtd_block_geometry(99, ctypes.byref(e), ctypes.byref(b)) == _lib.RTD_ERR_UNSUPPORTED
    assert b"99" in L.rtd_last_error(None)


def test_null_arguments_are_rejected_without_a_device():
    L = _lib.lib()
    assert L.rtd_init(0, None) == _lib.RTD_ERR_INVALID
    assert L.rtd_qlinear(None, None, None, 0, 0, 0, None, None, 0, 0, None) == _lib.RTD_ERR_INVALID
    assert L.rtd_destroy(None) == 0
    assert L.rtd_qweight_free(None) == 0


def test_init_fails_cleanly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert _lib.lib().rtd_init(0, ctypes.byref(h)) == _lib.RTD_ERR_CUDA
    assert not h.value


def test_noalloc_status_reader_reports_without_a_device():
    # the reader binds the device first: on a host without one it returns a CUDA error
    # (with a message on the calling thread) instead of touching memory
    L = _lib.lib()
    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("covered by the GPU tests")
    except ImportError:
        pass
    assert L.rtd_noalloc_check_status(0, None) == _lib.RTD_ERR_CUDA
    assert L.rtd_last_error(None)
    assert L.rtd_noalloc_check_status(-1, None) == _lib.RTD_ERR_INVALID


def test_entry_points_refuse_null_handles_without_a_device():
    # every compute entry point checks its handles before touching a device: NULL context or
    # weight is RTD_ERR_INVALID with a message, on any host
    L = _lib.lib()
    assert L.rtd_qlinear(None, None, None, 0, 1, 1, None, None, 0, 1, None) == _lib.RTD_ERR_INVALID
    assert L.rtd_qlinear_argmax(None, None, None, 0, 1, 1, None, None, 0, 1, None, None) == _lib.RTD_ERR_INVALID
    assert L.rtd_qlinear_argmax_keys(None, None, None, 0, 1, 1, None, 0, None, None) == _lib.RTD_ERR_INVALID
    assert L.rtd_argmax(None, None, 1, 1, 1, None, None) == _lib.RTD_ERR_INVALID
    assert L.rtd_qembed(None, None, None, 1, None, None) == _lib.RTD_ERR_INVALID
    assert L.rtd_last_error(None)
