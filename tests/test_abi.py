"""The C-ABI library loads and exports every function ``include/raon_cuda.h``
declares (CPU only: no function that needs a GPU is called)."""

import ctypes
import subprocess

import pytest

from raon_npu_b200 import _lib
from raon_npu_b200.build import LIB, build


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_header_declares_what_the_binding_declares():
    assert _lib.header_functions() == sorted(_lib.SIGNATURES)


def test_python_constants_match_the_header_defines():
    """Every ``#define RC_*`` integer of the header has the same value in the binding."""
    import re
    defines = dict(re.findall(r"^#define (RC_[A-Z0-9_]+) (\d+)u?\b", _lib.HEADER.read_text(), re.M))
    assert defines, "no integer defines found"
    for name, value in defines.items():
        assert getattr(_lib, name) == int(value), name


def test_library_exports_every_declared_symbol(lib):
    for name in _lib.header_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [n for n in _lib.header_functions() if n not in exported]
    assert not missing, missing


def test_library_has_no_torch_dependency():
    out = subprocess.run(["ldd", str(LIB)], capture_output=True, text=True).stdout
    # library names only: the load addresses in ldd's output are random hex
    names = [line.split()[0] for line in out.splitlines() if line.strip()]
    assert not any("torch" in n or "c10" in n for n in names), names


def test_abi_version_and_error_text(lib):
    assert lib.rc_abi_version() == 1
    assert isinstance(lib.rc_last_error(), bytes)


def test_argument_errors_raise_value_error_without_a_gpu(lib):
    # NULL out pointer is rejected before any CUDA call.
    assert lib.rc_init(0, None) == _lib.RC_ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(lib.rc_init(0, None))


def test_unknown_weight_handle_is_key_error(lib):
    n = ctypes.c_int()
    with pytest.raises(KeyError):
        _lib.check(lib.rc_weight_info(None, ctypes.byref(n), None, None, None))
