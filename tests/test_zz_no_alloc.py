"""clefq_gemm_noalloc: the quantized projection for callers that cannot allocate.

Some hosts cannot hand this library a workspace: a runtime that reserves all device memory
for its own allocator at start-up and passes a plugin only each call's inputs and outputs,
or an FFI binding without a workspace argument.  clefq_gemm_noalloc keeps its s8 operand
scratch in a fixed 64 MiB array of the library instead.  These tests call it through the
C ABI and require outputs identical to clefq_gemm with a caller workspace (the integer
GEMM is exact, so the tolerance is zero), on two calls in a row: BF16 and F32 outputs, a
BF16 residual, and a problem that fills the 64 MiB exactly.

This file is collected last on purpose (test_zz_*): a failure here stops a `-x` run only
after every other test has run.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as o
from tests.gpu_util import bf16_normal, from_dev_bf16, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu

LIMIT = 64 << 20  # CLEFQ_GEMM_NOALLOC_MAX_BYTES


def _call(lib, name, *args):
    rc = getattr(lib, name)(*args)
    assert rc == 0, f"{name}: {rc} {lib.clefq_last_error().decode()}"


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def cq():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import clefq
    clefq.lib()
    return clefq


def test_noalloc_warmup_call_then_real_call(cq):
    """m == 0 only loads and resolves the scratch array (what a host does on each device
    before its allocator reserves the memory); a real call afterwards works."""
    lib = cq.lib()
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _call(lib, "clefq_gemm_noalloc", s, None, 256 // 8, None, 0, None, None, 256, 256, None, 0, 0, None, 256)
    rng = np.random.default_rng(3)
    m, n, k = 40, 256, 512
    wt, ws = o.pack_weight(bf16_normal(rng, (n, k), 0.05))
    x = bf16_normal(rng, (m, k))
    a = cq.prepare(to_dev_bf16(x), 4, o.stride_for(k), operand=False)
    wt_d, ws_d = to_dev(wt.view(np.int32)), to_dev(ws)
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    _call(lib, "clefq_gemm_noalloc", s, _p(a.codes), a.codes.shape[1], _p(a.scales), m, _p(wt_d), _p(ws_d), n, k,
          None, 0, 0, _p(out), n)
    cq.status()
    _, ocodes, oscales, _ = o.prepare(x, 4, o.stride_for(k))
    assert np.array_equal(from_dev_bf16(out), o.gemm(ocodes, oscales, wt, ws, n, k))


@pytest.mark.parametrize("m,n,k,out_dtype,residual", [
    (300, 256, 1024, torch.bfloat16, False),
    (4096, 768, 4096, torch.bfloat16, False),
    (17, 384, 12288, torch.bfloat16, False),
    (300, 256, 1024, torch.float32, False),
    (513, 512, 2048, torch.float32, False),
    (300, 256, 1024, torch.bfloat16, True),
    (1000, 384, 4096, torch.bfloat16, True),
    (4096, 256, 16384, torch.bfloat16, False),   # m * k == 64 MiB: the whole scratch
])
def test_noalloc_matches_workspace_gemm(cq, m, n, k, out_dtype, residual):
    lib = cq.lib()
    rng = np.random.default_rng(m + n + k)
    w = bf16_normal(rng, (n, k), 0.05)
    wt, ws = o.pack_weight(w)
    x = bf16_normal(rng, (m, k))
    res = to_dev_bf16(bf16_normal(rng, (m, n))) if residual else None
    odt = 1 if out_dtype == torch.float32 else 0
    a = cq.prepare(to_dev_bf16(x), 4, o.stride_for(k), operand=False)
    wt_d, ws_d = to_dev(wt.view(np.int32)), to_dev(ws)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ref = torch.empty((m, n), dtype=out_dtype, device="cuda")
    need = lib.clefq_gemm_workspace_size(m, k, 4)
    ws_buf = torch.empty(need, dtype=torch.uint8, device="cuda")
    _call(lib, "clefq_gemm", s, 4, _p(a.codes), a.codes.shape[1], _p(a.scales), m, _p(wt_d), _p(ws_d), n, k, _p(res),
          n if residual else 0, odt, _p(ref), n, _p(ws_buf), need)
    outs = []
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
        _call(lib, "clefq_gemm_noalloc", s, _p(a.codes), a.codes.shape[1], _p(a.scales), m, _p(wt_d), _p(ws_d), n, k,
              _p(res), n if residual else 0, odt, _p(out), n)
        outs.append(out)
    torch.cuda.synchronize()
    cq.status()
    for out in outs:
        assert torch.equal(out.view(torch.int16 if odt == 0 else torch.int32),
                           ref.view(torch.int16 if odt == 0 else torch.int32))
    if m <= 300 and not residual and odt == 0:
        _, ocodes, oscales, _ = o.prepare(x, 4, o.stride_for(k))
        assert np.array_equal(from_dev_bf16(outs[1]), o.gemm(ocodes, oscales, wt, ws, n, k))


@pytest.mark.parametrize("m,k", [(8192, 16384), (LIMIT // 256 + 1, 256)])
def test_noalloc_rejects_oversized_problems(cq, m, k):
    """Twice the limit, and one 256-column row over it: CLEFQ_ERR_WORKSPACE before any
    pointer is touched."""
    lib = cq.lib()
    assert m * k > LIMIT
    rc = lib.clefq_gemm_noalloc(None, None, k // 8, None, m, None, None, 256, k, None, 0, 0, None, 256)
    assert rc == -6
    assert "64 MiB" in lib.clefq_last_error().decode()
