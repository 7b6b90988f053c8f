"""The drop-in boundary without a GPU: liborca_cuda.so loads, exports every
function include/orca_cuda.h declares, and the ctypes layer binds each one."""
import os

import pytest

from orcaml_b200 import _lib as L


def test_library_exports_every_declared_symbol():
    lib = L.load()
    syms = L.header_symbols()
    assert len(syms) >= 70
    missing = [s for s in syms if not hasattr(lib, s)]
    assert missing == []


def test_bindings_cover_the_header():
    assert sorted(set(L.header_symbols()) - set(L._SIGS)) == []
    assert sorted(set(L._SIGS) - set(L.header_symbols())) == []


def test_status_strings_and_version():
    lib = L.load()
    assert lib.orca_status_string(0) == b"ok"
    assert lib.orca_status_string(6) == b"timeout"
    assert lib.orca_version() >= 0x000100


def test_error_class_is_value_error():
    # The reference's PyO3 layer raises ValueError for every OrcaError.
    err = L.OrcaError(1, "x")
    assert isinstance(err, ValueError) and err.status_name == "ORCA_SHAPE_MISMATCH"
    assert issubclass(L.OrcaTimeout, L.OrcaError)


def test_library_is_sm100a_only_and_in_tree():
    assert os.path.dirname(L.LIB_PATH).endswith("orcaml_b200")
    with open(os.path.join(os.path.dirname(L.LIB_PATH), "build.py")) as f:
        assert "arch=compute_100a,code=sm_100a" in f.read()
