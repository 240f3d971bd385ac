"""CPU: the C-ABI library loads and exports every symbol the header declares."""

import ctypes

from utttcompanion_b200 import _lib


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    declared = _lib.header_symbols()
    assert declared, "no symbols parsed from include/uttt_b200.h"
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, missing
    # every declared symbol has a ctypes signature in the binding
    assert sorted(_lib.SIGNATURES) == declared


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.uttt_version() >= 1
    assert lib.uttt_status_string(0) == b"ok"
    assert b"timeout" in lib.uttt_status_string(4) or b"wait" in lib.uttt_status_string(4)


def test_invalid_arguments_rejected_on_host_without_gpu():
    lib = _lib.load()
    # NULL pointers and unsupported sizes are rejected before any CUDA call
    st = lib.uttt_selftest_gemm(0, 100, 64, 64, None, None, None, None, 0, None)
    assert st == _lib.UTTT_ERR_INVALID
    ws = ctypes.create_string_buffer(512)
    st = lib.uttt_selftest_gemm(0, 100, 64, 64, ctypes.addressof(ws), ctypes.addressof(ws),
                                ctypes.addressof(ws), ctypes.addressof(ws), 512, None)
    assert st == _lib.UTTT_ERR_UNSUPPORTED
