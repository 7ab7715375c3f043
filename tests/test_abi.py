"""The C-ABI library loads and exports every entry point include/clefq.h declares; host-side
argument checks reject bad shapes before touching a device (no GPU needed)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "clefq.h")).read()
    return sorted(set(re.findall(r"CLEFQ_API\s+[\w\s\*]+?\b(clefq_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    assert "clefq_gemm" in names and "clefq_moe" in names and len(names) >= 20


def test_library_exports_every_declared_symbol():
    import clefq
    lib = clefq.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) == set(clefq.exported_symbols())
    assert lib.clefq_version() >= 100


def test_workspace_queries():
    import clefq
    lib = clefq.lib()
    assert lib.clefq_gemm_workspace_size(128, 2048, 4) == 128 * 2048
    assert lib.clefq_gemm_workspace_size(128, 2048, 8) == 0
    assert lib.clefq_moe_workspace_size(8192, 2048, 768, 128, 8) > 8192 * 8 * 2048
    assert lib.clefq_mlp_workspace_size(4096, 4096, 12288) >= 4096 * 2 * 12288 * 2
    assert lib.clefq_expert_workspace_size(100, 8, 128, 2048) >= 800 * 2048


@pytest.mark.parametrize("args,msg", [
    ((0, 0, 3, None, 256, None, 0, 1, 256, 256, None, None, 0, None, 0), "bits"),
    ((0, 0, 4, None, 256, None, 0, 1, 300, 300, None, None, 0, None, 0), "width"),
    ((0, 0, 4, None, 256, None, 0, 0, 256, 256, None, None, 0, None, 0), "rows"),
    ((0, 0, 4, None, 256, None, 0, 1, 256, 200, None, None, 0, None, 0), "stride"),
])
def test_prepare_rejects_bad_shapes(args, msg):
    """src/quantized.rs:621-640 ensure! conditions become CLEFQ_ERR_SHAPE (-1)."""
    import clefq
    lib = clefq.lib()
    assert lib.clefq_prepare(*args) == -1
    assert msg in lib.clefq_last_error().decode()


def test_route_and_gemm_reject_bad_shapes():
    import clefq
    lib = clefq.lib()
    assert lib.clefq_route(None, None, 0, 4, 128, 0, None) == -1
    assert lib.clefq_route(None, None, 0, 4, 129, 8, None) == -1
    assert lib.clefq_gemm(None, 4, None, 256, None, 4, None, None, 100, 256, None, 0, 0, None, 100, None, 0) == -1
    assert lib.clefq_gemm(None, 4, None, 256, None, 4, None, None, 128, 300, None, 0, 0, None, 128, None, 0) == -1
    assert lib.clefq_retile(None, None, 100, 256, 4, 32, None) == -1
    assert lib.clefq_combine(None, None, None, None, 4, 8, 12, None) == -1


def test_python_api_rejects_cpu_tensors():
    import torch
    import clefq
    with pytest.raises(ValueError):
        clefq.prepare(torch.zeros(4, 256, dtype=torch.bfloat16))
