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


def _layout_ref(frames, ph, pw, rpf, v0, dense, keep):
    """src/models/h3.cpp:513-545 restated in numpy: cubes of 4 frames x 4 patch rows x 4 patch columns."""
    import math
    import numpy as np
    fc, yc, xc = -(-frames // 4), -(-ph // 4), -(-pw // 4)
    n = fc * yc * xc
    vrows = n * 64
    rows = vrows + dense
    q_pad, k_pad = -(-rows // 64) * 64, -(-rows // 128) * 128
    m = np.full(q_pad, -1, np.int32)
    valid = np.zeros(k_pad, np.uint8)
    cnt = np.zeros(n, np.uint32)
    for f in range(frames):
        for y in range(ph):
            for x in range(pw):
                cube = ((f // 4) * yc + y // 4) * xc + x // 4
                r = cube * 64 + ((f % 4) * 4 + y % 4) * 4 + x % 4
                m[r] = v0 + f * rpf + y * pw + x
                valid[r] = 1
                cnt[cube] += 1
    m[vrows:vrows + dense] = np.arange(dense)
    valid[vrows:vrows + dense] = 1
    return m, valid, cnt, dict(n_cubes=n, rows=rows, q_pad=q_pad, k_pad=k_pad, dense0=vrows, dense1=rows,
                               topk=max(1, math.ceil(keep * n)), stride=yc * xc)


@pytest.mark.parametrize("args", [(3, 10, 10, 100, 50, 50, 0.15), (21, 30, 30, 905, 7, 7, 0.25), (1, 1, 1, 1, 0, 0, 1.0),
                                  (5, 7, 9, 70, 3, 130, 0.5), (8, 12, 8, 96, 96, 96, 0.05)])
def test_cube_layout_matches_the_reference_loops(args):
    import numpy as np
    import mako_attn
    m, v, c, info = mako_attn.cube_layout(*args)
    wm, wv, wc, wi = _layout_ref(*args)
    np.testing.assert_array_equal(m, wm)
    np.testing.assert_array_equal(v, wv)
    np.testing.assert_array_equal(c, wc)
    for k, val in wi.items():
        assert getattr(info, k) == val, k


def test_cube_layout_rejections():
    import mako_attn
    with pytest.raises(mako_attn.MakoError, match="more than 4096 cubes"):
        mako_attn.cube_layout(68, 64, 64, 4096, 0, 0, 0.1)  # 17 x 16 x 16 = 4352 cubes
    with pytest.raises(mako_attn.MakoError, match="rows a frame"):
        mako_attn.cube_layout(2, 8, 8, 60, 0, 0, 0.1)
    with pytest.raises(mako_attn.MakoError, match="keep fraction"):
        mako_attn.cube_layout(2, 8, 8, 64, 0, 0, 0.0)
