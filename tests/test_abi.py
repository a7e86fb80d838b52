"""The C-ABI library builds for sm_100a, loads, and exports every entry point
declared in include/prism_bsa.h (no compute calls: these run without a GPU)."""
import ctypes
import os
import re

import pytest

from prism_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "prism_bsa.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(prism_[a-z0-9_]+)\s*\(",
                       src, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_path():
    names = declared_functions()
    for must in ("prism_zone_stats", "prism_shape_select", "prism_build_layout",
                 "prism_block_select", "prism_bsa_fwd", "prism_bsa_bwd", "prism_gather_rows",
                 "prism_scatter_rows", "prism_token_norms"):
        assert must in names


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    for name in declared_functions():
        assert hasattr(L, name), f"{name} not exported by {_lib.lib_path()}"
    assert set(declared_functions()) <= set(_lib.SIGNATURES), "ctypes table out of date"


def test_error_channel_without_gpu():
    L = _lib.load()
    assert L.prism_abi_version() >= 1
    # invalid arguments are rejected on the host before any CUDA call
    rc = L.prism_bsa_fwd(None, None, None, 1, 128, 128, ctypes.c_float(0.1), None, None, None,
                         None, None, None)
    assert rc != 0
    assert b"null pointer" in L.prism_last_error()
    rc = L.prism_shape_select(None, None, None, 0, 1, 64, 7, ctypes.c_float(0.5),
                              ctypes.c_float(0.15), ctypes.c_float(1.0), None, None, None, None)
    assert rc != 0
    rc = L.prism_copy_rows(None, 0, 256, None, 0, 256, 1, 4, 256, None)
    assert rc != 0 and b"null pointer" in L.prism_last_error()


def test_library_is_sm100a():
    # the fat binary carries sm_100a code only; checked through the build recipe
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)
    assert os.path.exists(build.LIB)
