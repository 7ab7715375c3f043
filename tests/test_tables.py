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


def _rne_bf16(bits):
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("err_steps", [0, 17, -17, 48, -48])
def test_silu_rounding_test_margin(err_steps):
    """The SwiGLU GEMM epilogue computes SiLU approximately and keeps the result only when
    Ziv's rounding test passes (silu_bf16_ziv, csrc/cq_common.cuh): q's f32 bits more than
    128 steps from a BF16 rounding midpoint, -16 < g < 8.  With the approximate quotient
    modelled as the float64 quotient moved by err_steps f32 steps (above the ~40-step error
    bound of the device expression), every kept value rounds to the table's entry; g >= 8
    gives g.  The GPU test of clefq_silu checks the device expression itself on all inputs."""
    tab = _table()
    g16 = np.arange(65536, dtype=np.uint32)
    g = (g16 << 16).view(np.float32).astype(np.float64)
    with np.errstate(over="ignore", invalid="ignore"):
        q = (g / (1.0 + np.exp(-g))).astype(np.float32)
    bits = q.view(np.uint32).astype(np.int64)
    bits = np.where(q != 0, bits + err_steps, bits).astype(np.uint32)
    margin = 128
    fast = (g > -16) & (g < 8) & (((bits.astype(np.int64) + margin - 0x8000) & 0xFFFF) > 2 * margin)
    assert fast.mean() > 0.5 * ((g > -16) & (g < 8)).mean()
    kept = np.nonzero(fast)[0]
    bad = kept[_rne_bf16(bits[kept].astype(np.int64)) != tab[kept]]
    assert bad.size == 0, [hex(int(i)) for i in bad[:8]]
    big = np.nonzero(np.isfinite(g) & (g >= 8) | (g16 == 0x7F80))[0]
    assert np.array_equal(tab[big], g16[big].astype(np.uint16))
