"""C-ABI checks that need no GPU: the library loads, exports exactly the symbols declared in
include/spinn_cuda.h, keeps the reference SpinnTensor layout, and rejects malformed .ennf
images on the host."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "spinn_cuda.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"\b(spinn_cuda_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    from spinn_b200 import lib
    L = lib.lib()
    for name in _declared():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted({ln.split()[-1] for ln in out.splitlines() if " T " in ln})
    assert exported == _declared()
    assert sorted(lib.declared_symbols()) == _declared()


def test_spinn_tensor_layout_matches_reference():
    from spinn_b200.lib import SpinnTensor
    assert ctypes.sizeof(SpinnTensor) == 72
    assert SpinnTensor.data.offset == 56 and SpinnTensor.size.offset == 44 and SpinnTensor.dims.offset == 4


def test_reference_tensor_layout(ref_oracle):
    assert ref_oracle.L.spinn_oracle_sizeof_tensor() == 72


def test_load_rejects_bad_images():
    from spinn_b200 import lib
    L = lib.lib()
    assert not L.spinn_cuda_load_buffer(b"\0" * 64, 64)
    assert "magic" in lib.last_error()
    assert not L.spinn_cuda_load_buffer(b"FNNE" + b"\0" * 10, 14)
    assert not L.spinn_cuda_load(b"/nonexistent/model.ennf")
    assert "cannot open" in lib.last_error()


def test_load_truncated_image():
    from spinn_b200 import ennf, lib, netdef
    g, _ = netdef.conv_bn_relu(hw=8, c=8, oc=8)
    img = ennf.convert(g)
    L = lib.lib()
    h = L.spinn_cuda_load_buffer(img, len(img))
    assert h
    L.spinn_cuda_free(h)
    bad = img[: len(img) // 3]
    assert not L.spinn_cuda_load_buffer(bad, len(bad))
    assert "truncated" in lib.last_error()


def test_run_before_plan_is_an_error():
    from spinn_b200 import ennf, lib, netdef
    g, _ = netdef.conv_bn_relu(hw=8, c=8, oc=8)
    img = ennf.convert(g)
    L = lib.lib()
    h = L.spinn_cuda_load_buffer(img, len(img))
    assert L.spinn_cuda_run(h, None, None) == lib.ESTATE
    assert L.spinn_cuda_io_count(h, 0) == 1 and L.spinn_cuda_io_count(h, 1) == 1
    dims = (ctypes.c_uint32 * 8)()
    assert L.spinn_cuda_io_dims(h, 1, 0, dims) == 4 and list(dims)[:4] == [1, 8, 8, 8]
    L.spinn_cuda_free(h)


def test_version_string():
    from spinn_b200 import lib
    assert b"sm_100a" in lib.lib().spinn_cuda_version()
