"""The C ABI without a GPU: the library loads, exports every symbol declared in
``include/cv3cuda.h``, and rejects bad arguments with the documented status
codes before touching the device."""

import ctypes
import os
import re

import pytest

from conftest import REPO, pkg

HEADER = os.path.join(REPO, "include", "cv3cuda.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*|unsigned long long)\s+(cv3_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    build = pkg("build")
    if not os.path.exists(build.LIB):
        build.build()
    return pkg("_lib").load()


def test_header_declares_the_abi():
    names = declared()
    assert "cv3_last_error" in names and "cv3_q8_linear" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), name


def test_host_binding_covers_every_declared_symbol():
    assert sorted(pkg("_lib").exported_names()) == declared()


def test_abi_version(lib):
    assert lib.cv3_abi_version() == 1


def test_bad_arguments_fail_before_any_device_work(lib):
    L = pkg("_lib")
    # padded K that is not a multiple of 64 -> CV3_ERR_VALUE with a message
    rc = lib.cv3_q8_linear(None, 1, 100, 100, None, None, 4, 100, None, None, None, 4, None)
    assert rc == L.CV3_ERR_VALUE
    assert b"padded K" in lib.cv3_last_error()
    with pytest.raises(ValueError, match="padded K"):
        L.check(rc, "cv3_q8_linear")
    # GQA head mismatch -> ValueError, the reference's exception for it
    rc = lib.cv3_attention(None, 0, 0, 0, None, 0, 0, 0, None, 0, 0, 0, None, 0, 0, 0,
                           1, 14, 3, 1, 1, 64, ctypes.c_float(0.125), 0, 0, 0, None)
    assert rc == L.CV3_ERR_VALUE
    assert b"not a multiple" in lib.cv3_last_error()
    # conv geometry mismatch
    rc = lib.cv3_conv1d(None, 1, 6, 10, None, 4, 3, 1, 1, 4, 0, 0, None, None, 8, None)
    assert rc == L.CV3_ERR_VALUE
    # unknown activation
    assert lib.cv3_unary(99, ctypes.c_float(0), None, 4, None, None) == L.CV3_ERR_VALUE


def test_zero_sized_calls_are_no_ops(lib):
    assert lib.cv3_q8_linear(None, 0, 64, 64, None, None, 8, 64, None, None, None, 8, None) == 0
    assert lib.cv3_unary(0, ctypes.c_float(0), None, 0, None, None) == 0
