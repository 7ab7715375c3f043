"""The BF16 SiLU table compiled into libclefq.so (clef-hrx_b200/csrc/gen_tables.cpp) equals
the oracle's SwiGLU activation for every BF16 input (kernels/swiglu.loom:41-50: the
activation is rounded to BF16 before the product, so with up = 1.0 the product is the
table entry itself)."""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "clef-hrx_b200")
TABLE = os.path.join(PKG, "_build", "silu_bf16.inc")


def _table():
    if not os.path.exists(TABLE):
        r = subprocess.run(["make", "-s", "-C", PKG, TABLE], capture_output=True, text=True)
        if r.returncode != 0:
            pytest.skip("table generator did not build: " + r.stderr[-200:])
    body = open(TABLE).read().split("\n", 1)[1]
    return np.array([int(t, 16) for t in body.replace(",", " ").split()], dtype=np.uint16)


def test_silu_table_matches_oracle_everywhere():
    tab = _table()
    assert tab.shape == (65536,)
    g = np.arange(65536, dtype=np.uint16)
    one = np.full(65536, 0x3F80, dtype=np.uint16)
    ref = O.swiglu(g, one).view(np.uint16)
    bad = np.nonzero(ref != tab)[0]
    assert bad.size == 0, [(hex(int(i)), hex(int(tab[i])), hex(int(ref[i]))) for i in bad[:8]]


def test_silu_table_known_values():
    tab = _table()
    # silu(0) = 0, silu(+inf) = +inf, silu(1) = 1/(1+e^-1) = 0.7310586 -> bf16 0x3f3b
    assert tab[0x0000] == 0x0000 and tab[0x8000] == 0x8000
    assert tab[0x7F80] == 0x7F80
    assert tab[0x3F80] == 0x3F3B
    # large negative inputs give -0 (g / inf)
    assert tab[0xC3C8] == 0x8000   # -400
