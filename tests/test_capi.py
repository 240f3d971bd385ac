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


def test_split_exchange_layout_and_host_checks_without_gpu():
    """The NVLink exchange area's size (flags [world][rows] u32 padded to 256 B, a 256-byte epoch
    word, two receive buffers [world][rows][d] FP32) and the host-side rejections of
    uttt_split_exchange_finish, none of which touches a GPU."""
    lib = _lib.load()
    world, rows, d = 8, 64, 2560
    flags = (world * rows * 4 + 255) // 256 * 256
    assert lib.uttt_split_exchange_bytes(world, rows, d) == flags + 256 + 2 * world * rows * d * 4
    assert lib.uttt_split_exchange_bytes(1, rows, d) == 0
    assert lib.uttt_split_exchange_bytes(9, rows, d) == 0
    buf = ctypes.create_string_buffer(512)
    p = ctypes.addressof(buf)
    areas = (ctypes.c_void_p * 2)(p, p)
    args = dict(rows=4, d=256, z=p, x=p, lw=p, lb=p, eps=1e-5, out=p, dt=_lib.DTYPE_BF16, zb=1, rank=0, world=2,
                max_rows=4, areas=ctypes.cast(areas, ctypes.c_void_p), polls=1 << 10, ws=p, wsb=512)

    def call(**kw):
        a = {**args, **kw}
        return lib.uttt_split_exchange_finish(a["rows"], a["d"], a["z"], a["x"], a["lw"], a["lb"], a["eps"],
                                              a["out"], a["dt"], a["zb"], a["rank"], a["world"], a["max_rows"],
                                              a["areas"], a["polls"], a["ws"], a["wsb"], None)
    assert call(rows=5) == _lib.UTTT_ERR_INVALID            # more rows than the areas hold
    assert call(world=9) == _lib.UTTT_ERR_INVALID           # at most 8 ranks
    assert call(rank=2) == _lib.UTTT_ERR_INVALID            # rank outside the group
    assert call(d=200) == _lib.UTTT_ERR_UNSUPPORTED         # d % 128 != 0
    assert call(wsb=16) == _lib.UTTT_ERR_WORKSPACE
    assert lib.uttt_ipc_alloc(0, None, None) == _lib.UTTT_ERR_INVALID
