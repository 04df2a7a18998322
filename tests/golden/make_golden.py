"""Writes tests/golden/sparse_attn_fixture.npz: the reference test's fixture (tests/sparse_attn_test.cpp:46-86 of
mako-common, re-created by the oracle with libstdc++'s normal_distribution) and the oracle's selection and attention
output on it (every 4th output row; the inputs by their SHA-256).  Run from the repository root: python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402


def main():
    O.build()
    fx = O.sparse_test_fixture()
    sel, nsel, *_ = O.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 3)
    sel_local, *_ = O.cube_select(0, fx["q"], fx["k"], 2, 448, 512, 6, fx["cnt"], 4, local=3, stride=1)
    o = np.full((448, 256), 12345.0, np.float32)
    O.attention_sparse(0, fx["q"], fx["k"], fx["v"], 444, 448, 444, 512, 2, 2, 256, 6, 3, 384, 444, sel, nsel,
                       fx["valid"], fx["map"], out=o)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sparse_attn_fixture.npz")
    rows = np.arange(0, 448, 4)
    sha = {"sha_" + n: hashlib.sha256(np.ascontiguousarray(fx[n]).tobytes()).hexdigest()
           for n in ("q", "k", "v", "valid", "map", "cnt")}
    np.savez_compressed(out, sel=sel, nsel=nsel, sel_local=sel_local, o_rows=rows, o_sub=o[rows], **sha)
    print(out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
