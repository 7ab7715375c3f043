"""clefq_gemm_noalloc: the quantized projection for callers that cannot allocate.

Some hosts cannot hand this library a workspace: a runtime that reserves all device memory
for its own allocator at start-up and passes a plugin only each call's inputs and outputs,
or an FFI binding without a workspace argument.  clefq_gemm_noalloc keeps its s8 operand
scratch in a fixed 64 MiB array of the library instead.  These tests call it through the
C ABI and require outputs identical to clefq_gemm with a caller workspace (the integer
GEMM is exact, so the tolerance is zero), on two calls in a row.

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


def _call(lib, name, *args):
    rc = getattr(lib, name)(*args)
    assert rc == 0, f"{name}: {rc} {lib.clefq_last_error().decode()}"


@pytest.mark.parametrize("m,n,k", [(300, 256, 1024), (4096, 768, 4096), (17, 384, 12288)])
def test_noalloc_matches_workspace_gemm(m, n, k):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import clefq
    lib = clefq.lib()
    rng = np.random.default_rng(m + n + k)
    w = bf16_normal(rng, (n, k), 0.05)
    wt, ws = o.pack_weight(w)
    x = bf16_normal(rng, (m, k))
    a = clefq.prepare(to_dev_bf16(x), 4, o.stride_for(k), operand=False)
    wt_d, ws_d = to_dev(wt.view(np.int32)), to_dev(ws)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ref = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    need = lib.clefq_gemm_workspace_size(m, k, 4)
    ws_buf = torch.empty(need, dtype=torch.uint8, device="cuda")
    _call(lib, "clefq_gemm", s, 4, ctypes.c_void_p(a.codes.data_ptr()), a.codes.shape[1],
          ctypes.c_void_p(a.scales.data_ptr()), m, ctypes.c_void_p(wt_d.data_ptr()), ctypes.c_void_p(ws_d.data_ptr()),
          n, k, None, 0, 0, ctypes.c_void_p(ref.data_ptr()), n, ctypes.c_void_p(ws_buf.data_ptr()), need)
    outs = []
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        _call(lib, "clefq_gemm_noalloc", s, ctypes.c_void_p(a.codes.data_ptr()), a.codes.shape[1],
              ctypes.c_void_p(a.scales.data_ptr()), m, ctypes.c_void_p(wt_d.data_ptr()),
              ctypes.c_void_p(ws_d.data_ptr()), n, k, None, 0, 0, ctypes.c_void_p(out.data_ptr()), n)
        outs.append(out)
    torch.cuda.synchronize()
    clefq.status()
    for out in outs:
        assert torch.equal(out, ref)
    if m <= 300:
        _, ocodes, oscales, _ = o.prepare(x, 4, o.stride_for(k))
        assert np.array_equal(from_dev_bf16(outs[1]), o.gemm(ocodes, oscales, wt, ws, n, k))


def test_noalloc_rejects_oversized_problems():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import clefq
    lib = clefq.lib()
    m, k = 8192, 16384  # 128 MiB of operand > 64 MiB
    rc = lib.clefq_gemm_noalloc(None, None, k // 8, None, m, None, None, 256, k, None, 0, 0, None, 256)
    assert rc == -6
    assert "64 MiB" in lib.clefq_last_error().decode()
