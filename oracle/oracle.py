"""clefq CPU oracle (TEST INFRASTRUCTURE ONLY) -- numpy front end over libclefq_oracle.so.

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module; the
product library never does.  Each function restates one reference operator; the C
source (clefq_oracle.c) cites the reference file:line for each.

Arrays: BF16 tensors are numpy uint16 bit patterns; packed codes are uint32 words; route,
group, order and task buffers are float32 exactly as in the reference.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libclefq_oracle.so")
_lib = None

PLAIN, SWIGLU, ATTN_GATE, NORM, NORM_STORE = 0, 1, 2, 3, 4


def build() -> str:
    """Compile the oracle shared library in place (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        _lib.cqo_prepare.argtypes = [i32, i32, vp, i64, vp, i64, i64, i64, i64, vp, vp, i64, i32]
        _lib.cqo_retile.argtypes = [vp, i64, i64, i64, vp]
        _lib.cqo_gemm.argtypes = [i32, vp, i64, vp, i64, vp, vp, i64, i64, vp, i32, vp, vp, i32]
        _lib.cqo_swiglu.argtypes = [vp, vp, i64, vp, i32]
        _lib.cqo_route.argtypes = [vp, i32, i64, i32, i32, vp, i32]
        _lib.cqo_group.argtypes = [vp, i64, i32, i32, vp, vp]
        _lib.cqo_tasks.argtypes = [vp, i64, i32, vp]
        _lib.cqo_expert.argtypes = [i32, vp, i64, vp, vp, vp, vp, i64, i32, i32, i64, i64, i32, vp, i32]
        _lib.cqo_combine.argtypes = [vp, vp, vp, i64, i32, i64, vp, i32]
        _lib.cqo_exp.argtypes = [vp, i64, vp]
        for name in ("cqo_prepare", "cqo_retile", "cqo_gemm", "cqo_route", "cqo_group", "cqo_tasks",
                     "cqo_expert", "cqo_combine"):
            getattr(_lib, name).restype = ctypes.c_int
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def _check(rc, what):
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments (status {rc})")


# ---------------------------------------------------------------------------------------
# BF16 helpers (round to nearest even; NaN keeps sign, quiet bit forced)
# ---------------------------------------------------------------------------------------
def f32_to_bf16(x) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def stride_for(k: int, bits: int = 4) -> int:
    """Activation/weight row pitch in codes (src/quantized.rs:154-166)."""
    return k + (512 // bits if k % 1024 == 0 else 0)


# ---------------------------------------------------------------------------------------
# Operators
# ---------------------------------------------------------------------------------------
def prepare(x, bits=4, stride=None, mode=PLAIN, aux=None, threads=None):
    """Hadamard-256 + per-row quantization.  Returns (storage u32, codes view, scales view,
    norm_out or None) with storage = codes[rows][stride/P] then f32 scales[rows]."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    rows, width = x.shape
    stride = stride_for(width, bits) if stride is None else stride
    words = stride // (32 // bits)
    storage = np.zeros(rows * (words + 1), dtype=np.uint32)
    norm_out = np.zeros((rows, width), dtype=np.uint16) if mode == NORM_STORE else None
    aux_ld = 0
    if aux is not None:
        aux = np.ascontiguousarray(aux, dtype=np.uint16)
        aux_ld = aux.shape[-1] if aux.ndim == 2 else 0
    rc = lib().cqo_prepare(mode, bits, _p(x), width, _p(aux), aux_ld, rows, width, stride, _p(storage),
                           _p(norm_out), width, threads or default_threads())
    _check(rc, "prepare")
    codes = storage[: rows * words].reshape(rows, words)
    scales = storage[rows * words:].view(np.float32)
    return storage, codes, scales, norm_out


def retile(codes, rows, cols, bits=4):
    codes = np.ascontiguousarray(codes, dtype=np.uint32)
    words = cols // (32 // bits)
    out = np.zeros(rows * words, dtype=np.uint32)
    _check(lib().cqo_retile(_p(codes), rows, codes.shape[-1], words, _p(out)), "retile")
    return out


def pack_weight(w_bf16, bits=4, threads=None):
    """load_quantized_weight (src/quantized.rs:147-234) minus the checkpoint untiling:
    prepare (weights rotated and quantized like activations), retile, compact scales."""
    rows, cols = w_bf16.shape
    stride = stride_for(cols, bits)
    _, codes, scales, _ = prepare(w_bf16, bits, stride, threads=threads)
    return retile(codes, rows, cols, bits), scales.copy()


def gemm(a_codes, a_scales, w_tiled, w_scales, n, k, bits=4, residual=None, out_f32=False, want_acc=False,
         threads=None):
    a_codes = np.ascontiguousarray(a_codes, dtype=np.uint32)
    m = a_codes.shape[0]
    out = np.zeros((m, n), dtype=np.float32 if out_f32 else np.uint16)
    acc = np.zeros((m, n), dtype=np.int32) if want_acc else None
    res = None if residual is None else np.ascontiguousarray(residual, dtype=np.uint16)
    rc = lib().cqo_gemm(bits, _p(a_codes), a_codes.shape[1], _p(np.ascontiguousarray(a_scales, np.float32)), m,
                        _p(np.ascontiguousarray(w_tiled, np.uint32)), _p(np.ascontiguousarray(w_scales, np.float32)),
                        n, k, _p(res), int(out_f32), _p(out), _p(acc), threads or default_threads())
    _check(rc, "gemm")
    return (out, acc) if want_acc else out


def swiglu(g, u, threads=None):
    g = np.ascontiguousarray(g, dtype=np.uint16)
    u = np.ascontiguousarray(u, dtype=np.uint16)
    out = np.zeros_like(g)
    lib().cqo_swiglu(_p(g), _p(u), g.size, _p(out), threads or default_threads())
    return out


def route(logits, topk=8, threads=None):
    logits = np.ascontiguousarray(logits)
    tokens, experts = logits.shape
    is_f32 = logits.dtype == np.float32
    if not is_f32:
        logits = logits.astype(np.uint16)
    out = np.zeros((tokens, 2 * topk), dtype=np.float32)
    _check(lib().cqo_route(_p(logits), int(is_f32), tokens, experts, topk, _p(out), threads or default_threads()),
           "route")
    return out


def group(routes, experts=128):
    routes = np.ascontiguousarray(routes, dtype=np.float32)
    tokens, width = routes.shape
    topk = width // 2
    groups = np.zeros((experts, tokens + 1), dtype=np.float32)
    order = np.zeros((tokens, topk), dtype=np.float32)
    lib().cqo_group(_p(routes), tokens, topk, experts, _p(groups), _p(order))
    return groups, order


def tasks(groups, tokens, topk=8, experts=128):
    n = 1 + 2 * (-(-tokens * topk // 16) + experts - 1)
    out = np.zeros(n, dtype=np.float32)
    lib().cqo_tasks(_p(np.ascontiguousarray(groups, np.float32)), tokens, experts, _p(out))
    return out


def expert(a_codes, a_scales, w_tiled, w_scales, groups, tokens, k, n, input_routed, topk=8, experts=128,
           threads=None):
    a_codes = np.ascontiguousarray(a_codes, dtype=np.uint32)
    out = np.zeros((tokens * topk, n), dtype=np.uint16)
    rc = lib().cqo_expert(4, _p(a_codes), a_codes.shape[1], _p(np.ascontiguousarray(a_scales, np.float32)),
                          _p(np.ascontiguousarray(w_tiled, np.uint32)),
                          _p(np.ascontiguousarray(w_scales, np.float32)),
                          _p(np.ascontiguousarray(groups, np.float32)), tokens, topk, experts, k, n,
                          int(input_routed), _p(out), threads or default_threads())
    _check(rc, "expert")
    return out


def combine(values, routes, order=None, threads=None):
    values = np.ascontiguousarray(values, dtype=np.uint16)
    routes = np.ascontiguousarray(routes, dtype=np.float32)
    tokens, width2 = routes.shape
    topk = width2 // 2
    width = values.shape[1]
    out = np.zeros((tokens, width), dtype=np.uint16)
    o = None if order is None else np.ascontiguousarray(order, dtype=np.float32)
    lib().cqo_combine(_p(values), _p(routes), _p(o), tokens, topk, width, _p(out), threads or default_threads())
    return out


def exp(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros_like(x)
    lib().cqo_exp(_p(x), x.size, _p(out))
    return out


# ---------------------------------------------------------------------------------------
# Composite paths (the timed CPU baselines)
# ---------------------------------------------------------------------------------------
def mlp_block(x, gate, up, down, threads=None):
    """Dense INT4 SwiGLU MLP (the reference's generic route, src/quantized.rs:406-439 with
    src/backbone.rs:880-894): prepare(x) -> gate, up -> SwiGLU -> prepare -> down.
    gate/up/down are (tiled codes, scales, rows, cols)."""
    m, h = x.shape
    _, codes, scales, _ = prepare(x, 4, stride_for(h), threads=threads)
    g = gemm(codes, scales, gate[0], gate[1], gate[2], h, threads=threads)
    u = gemm(codes, scales, up[0], up[1], up[2], h, threads=threads)
    hid = swiglu(g, u, threads=threads)
    inter = hid.shape[1]
    _, hc, hs, _ = prepare(hid, 4, stride_for(inter), threads=threads)
    return gemm(hc, hs, down[0], down[1], down[2], inter, threads=threads)


def normalized_mlp_block(x, norm_w, gate, up, down, threads=None):
    """Pre-norm MLP with the input as residual (src/quantized.rs:348-404): RMSNorm fused into
    the packing of x (prepare_norm_with_source), gate, up, SwiGLU, packing, down + x."""
    m, h = x.shape
    _, codes, scales, _ = prepare(x, 4, stride_for(h), NORM, norm_w, threads=threads)
    g = gemm(codes, scales, gate[0], gate[1], gate[2], h, threads=threads)
    u = gemm(codes, scales, up[0], up[1], up[2], h, threads=threads)
    hid = swiglu(g, u, threads=threads)
    inter = hid.shape[1]
    _, hc, hs, _ = prepare(hid, 4, stride_for(inter), threads=threads)
    return gemm(hc, hs, down[0], down[1], down[2], inter, residual=x, threads=threads)


def moe_layer(x, logits, gate, up, down, topk=8, experts=128, threads=None):
    """Omni INT4 MoE block (src/omni.rs:761-857 with fast defaults): route -> ordered groups
    -> gate, up experts (shared packing) -> SwiGLU -> down experts -> ordered combine."""
    tokens, hidden = x.shape
    routes = route(logits, topk, threads=threads)
    groups, order = group(routes, experts)
    _, xc, xs, _ = prepare(x, 4, stride_for(hidden), threads=threads)
    inter = gate[2]
    g = expert(xc, xs, gate[0], gate[1], groups, tokens, hidden, inter, False, topk, experts, threads)
    u = expert(xc, xs, up[0], up[1], groups, tokens, hidden, inter, False, topk, experts, threads)
    hid = swiglu(g, u, threads=threads)
    _, hc, hs, _ = prepare(hid, 4, stride_for(inter), threads=threads)
    vals = expert(hc, hs, down[0], down[1], groups, tokens, inter, hidden, True, topk, experts, threads)
    return combine(vals, routes, order, threads=threads), routes, groups, order
