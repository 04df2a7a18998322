"""The C ABI library loads and exports every function include/mako_attn.h declares; host-side argument handling
that needs no GPU (no compute is called here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mako_attn.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mako_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for want in ("mako_attention", "mako_attention_decode", "mako_cube_select", "mako_attention_sparse",
                 "mako_attn_create", "mako_attn_destroy", "mako_attn_last_error"):
        assert want in names


def test_library_exports_every_declared_symbol():
    import mako_attn
    L = mako_attn.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert set(mako_attn.SYMBOLS) == set(declared_functions())
    assert L.mako_attn_version() == 1


def test_null_context_is_rejected_before_any_launch():
    import mako_attn
    L = mako_attn.lib()
    rc = L.mako_attention(None, None, 0, None, None, None, None, 1, 64, 1, 128, 1, 1, 0, 0, 128, 0)
    assert rc == mako_attn.EINVAL
    assert b"context" in L.mako_attn_last_error()
    sel, nsel = ctypes.c_void_p(), ctypes.c_void_p()
    rc = L.mako_cube_select(None, None, 0, None, None, 1, 64, 128, 1, None, 1, ctypes.byref(sel), ctypes.byref(nsel),
                            0, 0)
    assert rc == mako_attn.EINVAL


def test_create_without_a_device_reports_the_cuda_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    import mako_attn
    L = mako_attn.lib()
    h = ctypes.c_void_p()
    rc = L.mako_attn_create(0, ctypes.byref(h))
    assert rc in (mako_attn.ECUDA, mako_attn.EINVAL) and not h.value
    assert L.mako_attn_last_error()


def test_cpp_shim_compiles_links_and_throws(tmp_path):
    """include/mako_attn.hpp over libmako_attn.so: a bad call (or no device) surfaces as std::runtime_error."""
    import subprocess
    lib_dir = os.path.join(ROOT, "mako-common_b200", "mako_attn")
    exe = str(tmp_path / "shim_check")
    subprocess.run(["/usr/bin/g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "shim_check.cpp"), "-L", lib_dir, "-lmako_attn",
                    f"-Wl,-rpath,{lib_dir}", "-o", exe], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
