"""The C ABI surface of libnufft_b200.so: every symbol declared in
include/nufft_b200.h is exported, the ctypes layouts match the C structs,
and the entry points report errors by status code without a GPU."""

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from mlx_nufft_b200 import _lib
from mlx_nufft_b200._lib import lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nufft_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nufft_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    names = declared_functions()
    assert len(names) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (nufft_[a-z0-9_]+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # and the Python binding covers every one of them
    assert set(names) == set(_lib.EXPORTED)


def test_struct_layouts_match_header(tmp_path):
    prog = tmp_path / "sz.c"
    prog.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "nufft_b200.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu\\n\", sizeof(nufft_opts),"
        " sizeof(nufft_plan_info), offsetof(nufft_plan_info, device_bytes),"
        " offsetof(nufft_opts, source_extent));return 0;}\n")
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(prog), "-o",
                    str(exe)], check=True)
    vals = [int(v) for v in subprocess.run([str(exe)], capture_output=True,
                                           text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(_lib.NufftOpts)
    assert vals[1] == ctypes.sizeof(_lib.NufftPlanInfo)
    assert vals[2] == _lib.NufftPlanInfo.device_bytes.offset
    assert vals[3] == _lib.NufftOpts.source_extent.offset


def test_default_opts():
    o = _lib.default_opts()
    assert o.prec == 0 and o.method == 0 and o.sort_points == 1
    assert o.upsampfac == 0.0 and o.max_batch == 0 and o.profile == 0


def test_version_and_device_count():
    assert b"sm_100a" in lib.nufft_version()
    assert lib.nufft_device_count() >= 0


def test_argument_errors_are_status_codes():
    h = ctypes.c_void_p()
    nm = (ctypes.c_int64 * 3)(8, 8, 8)
    rc = lib.nufft_plan_create(4, 1, nm, 1, 1e-6, 1, None, 0, ctypes.byref(h))
    assert rc == _lib.NUFFT_ERR_ARG
    assert "nufft_type" in _lib.last_error()
    rc = lib.nufft_plan_create(1, 0, nm, 1, 1e-6, 1, None, 0, ctypes.byref(h))
    assert rc == _lib.NUFFT_ERR_ARG
    rc = lib.nufft_plan_create(1, 1, nm, 0, 1e-6, 1, None, 0, ctypes.byref(h))
    assert rc == _lib.NUFFT_ERR_ARG
    rc = lib.nufft_plan_create(1, 1, nm, 1, -1.0, 1, None, 0, ctypes.byref(h))
    assert rc == _lib.NUFFT_ERR_ARG
    assert lib.nufft_execute(None, None, None, 1, None) == _lib.NUFFT_ERR_ARG
    assert lib.nufft_setpts(None, 1, None, None, None, 0, None, None, None,
                            None) == _lib.NUFFT_ERR_ARG
    assert lib.nufft_plan_destroy(None) == 0
    with pytest.raises(ValueError):
        _lib.check(_lib.NUFFT_ERR_ARG)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.NUFFT_ERR_STATE)
    with pytest.raises(MemoryError):
        _lib.check(_lib.NUFFT_ERR_OOM)


@pytest.mark.skipif(lib.nufft_device_count() > 0, reason="GPU present")
def test_plan_create_without_gpu_fails_loudly():
    h = ctypes.c_void_p()
    nm = (ctypes.c_int64 * 3)(8, 1, 1)
    rc = lib.nufft_plan_create(1, 1, nm, 1, 1e-6, 1, None, 0, ctypes.byref(h))
    assert rc == _lib.NUFFT_ERR_CUDA
    assert "no CUDA device" in _lib.last_error()


def test_expi_argument_errors():
    arr = (ctypes.c_void_p * 1)(None)
    assert lib.nufft_expi(1, None, 10, 1, None, None) == _lib.NUFFT_ERR_ARG
    assert lib.nufft_expi(1, arr, 10, 1, None, None) == _lib.NUFFT_ERR_ARG
