"""The C-ABI library builds, loads without a GPU, and exports exactly the
symbols include/bsgpu.h declares (no compute calls here)."""
from __future__ import annotations

import os
import re
import subprocess

from tests.conftest import ROOT


def _declared():
    hdr = open(os.path.join(ROOT, "include", "bsgpu.h")).read()
    return set(re.findall(r"^(?:int|const char \*)\s*(bs_\w+)\(", hdr, re.M))


def test_header_declarations_match_binding():
    from bigsmall_b200 import _lib
    assert _declared() == set(_lib.SIGNATURES)


def test_library_loads_and_exports_every_symbol():
    from bigsmall_b200 import _lib
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    assert lib.bs_version() == 101
    assert lib.bs_status_string(5) == b"corrupt stream"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (bs_\w+)", out))
    assert _declared() <= exported
    # measurement tooling lives in its own library, outside the product ABI
    assert "bs_stream_probe" not in exported
    calib = os.path.join(os.path.dirname(_lib.LIB_PATH), "libbscalib.so")
    out = subprocess.run(["nm", "-D", "--defined-only", calib], capture_output=True, text=True).stdout
    assert re.findall(r" T (bs_\w+)", out) == ["bs_stream_probe"]


def test_host_side_validation_without_gpu():
    """Argument checks run before any device work."""
    import ctypes
    from bigsmall_b200 import _lib
    lib = _lib.load()
    v = ctypes.c_uint64()
    assert lib.bs_xc_encode_bound(1000, 100, 1, ctypes.byref(v)) == _lib.BS_E_INVALID_ARG
    assert lib.bs_xc_encode_bound(1000, 256, 1, ctypes.byref(v)) == 0 and v.value > 2000
    assert lib.bs_xc_encode_bound(1000, 256, 0, ctypes.byref(v)) == 0      # 0 groups: one
    # chunk_elems / groups must be a positive multiple of 256
    for ce, g, ok in ((8192, 4, True), (8192, 3, False), (1024, 8, False), (1 << 22, 128, True)):
        assert (lib.bs_xc_encode_bound(1000, ce, g, ctypes.byref(v)) == 0) == ok, (ce, g)
    for coder, ok in ((0, True), (1, True), (2, True), (3, False), (-1, False)):
        rc = lib.bs_xc_encode_workspace(100_000, 4096, 1, coder, ctypes.byref(v))
        assert (rc == 0) == ok, coder
    h = ctypes.c_void_p()
    # no CUDA device in a CPU-only container: creation must fail cleanly
    rc = lib.bs_xc_plan_create(None, 0, 0, ctypes.byref(h))
    assert rc in (_lib.BS_OK, _lib.BS_E_INVALID_ARG)
    if rc == _lib.BS_OK:
        lib.bs_plan_destroy(h)


def test_ctypes_mirrors_match_the_c_layout(tmp_path):
    """The ctypes mirrors of the ABI's structs have the C compiler's size and
    field offsets (a stale mirror would mis-stride descriptor arrays)."""
    import ctypes
    from bigsmall_b200 import _lib
    structs = {"bs_xc_tensor": _lib.XcTensor, "bs_se_blob": _lib.SeBlob}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "bsgpu.h"', 'int main(void) {']
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["return 0; }"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(py, f).offset, (cname, f)
