"""The C ABI: libb200.so builds for sm_100a, loads without a GPU and exports exactly
the entry points include/b200.h declares (no compute call is made here)."""

import os
import re

from conftest import ROOT


def declared_symbols():
    hdrs = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h")]
    names = set()
    for h in hdrs:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[\w\s\*]+?\b(b200_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("b200_ew_run", "b200_gemm", "b200_softmax", "b200_layernorm", "b200_conv2d_fwd", "b200_argmax"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from b200 import _lib as L
    from b200.build import build

    build()
    lib = L.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.b200_abi_version() == 1
    # every declared symbol has a ctypes signature in the shim
    assert declared_symbols() <= set(L.SIGNATURES), declared_symbols() - set(L.SIGNATURES)


def test_ew_program_struct_layout():
    import ctypes

    from b200 import _lib as L

    # int32 x4, int64[6], int64[8][6], int32[8], int32[4], ins[48] x 12 bytes
    assert ctypes.sizeof(L.EwIns) == 12
    expected = 16 + 48 + 384 + 32 + 16 + 48 * 12
    assert ctypes.sizeof(L.EwProgram) == expected
