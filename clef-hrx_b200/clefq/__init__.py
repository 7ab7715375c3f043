"""clefq -- host-side mirror of clef-hrx's INT4 quantized-matmul API over the C ABI.

Names, argument meaning and error behaviour follow the reference's Rust operators
(src/quantized.rs, src/omni.rs, src/ops.rs): shape violations raise ValueError (the
reference's `ensure!`), device failures raise RuntimeError.  Every call goes through
libclefq.so (include/clefq.h); PyTorch only provides device memory and the current
stream.  There is no CPU fallback: importing this package without the built library
raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libclefq.so")

PREP_PLAIN, PREP_SWIGLU, PREP_ATTN_GATE, PREP_NORM, PREP_NORM_STORE = 0, 1, 2, 3, 4
BF16, F32, ROUTER_WEIGHT_BF16 = 0, 1, 2
EXPERTS, TOP_K = 128, 8

ERRORS = {-1: "shape", -2: "alignment", -3: "cuda", -4: "nccl", -5: "timeout", -6: "workspace"}

_SYMBOLS = {
    # name: (restype, argtypes)
    "clefq_last_error": (ctypes.c_char_p, []),
    "clefq_version": (ctypes.c_int, []),
    "clefq_status": (ctypes.c_int, ["p"]),
    "clefq_prepare": (ctypes.c_int, ["p", "i", "i", "p", "l", "p", "l", "l", "l", "l", "p", "p", "l", "p", "l"]),
    "clefq_retile": (ctypes.c_int, ["p", "p", "l", "l", "i", "l", "p"]),
    "clefq_gemm_workspace_size": (ctypes.c_int64, ["l", "l", "i"]),
    "clefq_gemm": (ctypes.c_int, ["p", "i", "p", "l", "p", "l", "p", "p", "l", "l", "p", "l", "i", "p", "l", "p", "l"]),
    "clefq_gemm_s8": (ctypes.c_int, ["p", "i", "p", "l", "p", "l", "p", "p", "l", "l", "p", "l", "i", "p", "l"]),
    "clefq_gemm_noalloc": (ctypes.c_int, ["p", "p", "l", "p", "l", "p", "p", "l", "l", "p", "l", "i", "p", "l"]),
    "clefq_gemm_pair_s8": (ctypes.c_int, ["p", "p", "l", "p", "l", "p", "p", "p", "p", "l", "l", "p", "l"]),
    "clefq_gemm_swiglu_s8": (ctypes.c_int, ["p", "p", "l", "p", "l", "p", "p", "p", "p", "l", "l", "p", "l"]),
    "clefq_swiglu": (ctypes.c_int, ["p", "p", "p", "l", "p"]),
    "clefq_silu": (ctypes.c_int, ["p", "p", "l", "p"]),
    "clefq_route": (ctypes.c_int, ["p", "p", "i", "l", "i", "i", "p"]),
    "clefq_route_linear": (ctypes.c_int, ["p", "p", "p", "l", "l", "i", "i", "p", "p"]),
    "clefq_group_workspace_size": (ctypes.c_int64, ["l", "i", "i"]),
    "clefq_group_routes": (ctypes.c_int, ["p", "p", "l", "i", "i", "p", "p", "p", "l"]),
    "clefq_expert_tasks": (ctypes.c_int, ["p", "p", "l", "i", "p"]),
    "clefq_expert_workspace_size": (ctypes.c_int64, ["l", "i", "i", "l"]),
    "clefq_expert": (ctypes.c_int, ["p", "p", "l", "p", "p", "p", "p", "l", "i", "i", "l", "l", "i", "p", "p", "l"]),
    "clefq_expert_gate_up": (ctypes.c_int, ["p", "p", "l", "p", "p", "p", "p", "p", "p", "l", "i", "i", "l", "l", "p",
                                            "p", "l"]),
    "clefq_combine": (ctypes.c_int, ["p", "p", "p", "p", "l", "i", "l", "p"]),
    "clefq_mlp_workspace_size": (ctypes.c_int64, ["l", "l", "l"]),
    "clefq_mlp": (ctypes.c_int, ["p", "p", "l", "l", "l", "p", "p", "p", "p", "p", "p", "p", "p", "p", "l"]),
    "clefq_normalized_mlp": (ctypes.c_int, ["p", "p", "l", "l", "l", "p", "p", "p", "p", "p", "p", "p", "p", "p",
                                            "l"]),
    "clefq_mlp_host_workspace_size": (ctypes.c_int64, ["l", "l", "l", "i"]),
    "clefq_mlp_host": (ctypes.c_int, ["p", "p", "l", "l", "l", "p", "p", "p", "p", "p", "p", "p", "p", "l", "i", "p",
                                      "p", "l"]),
    "clefq_moe_workspace_size": (ctypes.c_int64, ["l", "l", "l", "i", "i"]),
    "clefq_moe": (ctypes.c_int, ["p", "p", "p", "i", "l", "l", "l", "i", "i", "p", "p", "p", "p", "p", "p", "p", "p",
                                 "p", "l"]),
    "clefq_moe_ep_record_bytes": (ctypes.c_int64, ["l"]),
    "clefq_moe_ep_plan_workspace_size": (ctypes.c_int64, ["i"]),
    "clefq_moe_ep_plan": (ctypes.c_int, ["p", "p", "l", "i", "i", "i", "p", "p", "p", "l"]),
    "clefq_moe_ep_pack": (ctypes.c_int, ["p", "p", "l", "p", "l", "l", "p", "i", "p", "p"]),
    "clefq_moe_ep_experts_workspace_size": (ctypes.c_int64, ["l", "l", "l", "i"]),
    "clefq_moe_ep_experts": (ctypes.c_int, ["p", "p", "l", "l", "l", "i", "i", "p", "p", "p", "p", "p", "p", "p", "p",
                                            "l"]),
    "clefq_moe_ep_combine": (ctypes.c_int, ["p", "p", "p", "p", "l", "i", "l", "p"]),
    "clefq_prepare_rowmax": (ctypes.c_int, ["p", "i", "p", "l", "p", "l", "l", "l", "p"]),
    "clefq_prepare_scaled": (ctypes.c_int, ["p", "i", "i", "p", "l", "p", "l", "l", "l", "l", "p", "p", "p", "l"]),
    "clefq_tp_gather_unpack": (ctypes.c_int, ["p", "p", "i", "l", "l", "p", "l"]),
    "clefq_tp_interleave": (ctypes.c_int, ["p", "p", "i", "l", "l", "p", "l"]),
    "clefq_comm_handle_bytes": (ctypes.c_int64, []),
    "clefq_comm_create": (ctypes.c_int, ["i", "i", "l", "p", "p"]),
    "clefq_comm_open": (ctypes.c_int, ["p", "p"]),
    "clefq_comm_attach": (ctypes.c_int, ["p", "i", "p"]),
    "clefq_comm_ready": (ctypes.c_int, ["p"]),
    "clefq_comm_region": (ctypes.c_void_p, ["p"]),
    "clefq_comm_region_bytes": (ctypes.c_int64, ["p"]),
    "clefq_comm_set_timeout_ms": (ctypes.c_int, ["p", "l"]),
    "clefq_comm_barrier": (ctypes.c_int, ["p", "p"]),
    "clefq_comm_destroy": (ctypes.c_int, ["p"]),
    "clefq_tp_mlp_region_bytes": (ctypes.c_int64, ["l", "l", "l", "i"]),
    "clefq_tp_mlp_workspace_size": (ctypes.c_int64, ["l", "l", "l", "i"]),
    "clefq_tp_mlp": (ctypes.c_int, ["p", "p", "p", "l", "l", "l", "p", "p", "p", "p", "p", "p", "p", "p", "p", "l"]),
    "clefq_tp_mlp_output": (ctypes.c_void_p, ["p", "l", "l", "l"]),
    "clefq_untile_bf16": (ctypes.c_int, ["p", "p", "l", "l", "p"]),
    "clefq_load_weight_workspace_size": (ctypes.c_int64, ["l", "l", "i", "i"]),
    "clefq_load_weight": (ctypes.c_int, ["p", "p", "l", "l", "i", "i", "p", "p", "p", "l"]),
    "clefq_moe_ep_layer_region_bytes": (ctypes.c_int64, ["l", "l", "i", "i", "l"]),
    "clefq_moe_ep_layer_workspace_size": (ctypes.c_int64, ["l", "l", "l", "i", "i", "i", "l"]),
    "clefq_moe_ep_layer": (ctypes.c_int, ["p", "p", "p", "p", "i", "l", "l", "l", "i", "i", "l", "p", "p", "p", "p", "p",
                                          "p", "p", "p", "p", "l"]),
}
_CT = {"p": ctypes.c_void_p, "i": ctypes.c_int, "l": ctypes.c_int64}

_lib = None


def lib():
    """Load libclefq.so (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"clefq: {LIB_PATH} is missing; build it with `make -C clef-hrx_b200` "
                               "or __graft_entry__.build()")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SYMBOLS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = [_CT[a] for a in args]
        _lib = handle
    return _lib


def exported_symbols():
    return list(_SYMBOLS)


def _call(name, *args):
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        msg = lib().clefq_last_error().decode(errors="replace")
        if rc == -1:
            raise ValueError(f"{name}: {msg}")
        raise RuntimeError(f"{name} failed ({ERRORS.get(rc, rc)}): {msg}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("clefq operates on CUDA tensors")


def stride_for(cols: int, bits: int = 4) -> int:
    """Row pitch in codes (src/quantized.rs:154-166)."""
    return cols + (512 // bits if cols % 1024 == 0 else 0)


def status():
    """Synchronize and raise if a bounded device-side wait gave up since the last check."""
    _call("clefq_status", _stream())


# ---------------------------------------------------------------------------------------
# Packing (src/quantized.rs:574-776)
# ---------------------------------------------------------------------------------------
@dataclass
class Prepared:
    storage: torch.Tensor   # int32 [rows*(words+1)]: codes then f32 scales
    codes: torch.Tensor     # int32 view [rows][words]
    scales: torch.Tensor    # float32 view [rows]
    operand: torch.Tensor | None  # int8 [rows][width] GEMM operand (bits 4)
    norm: torch.Tensor | None     # bf16 [rows][width] (norm_store)
    bits: int
    stride: int


def prepare(x, bits=4, stride=None, kind=PREP_PLAIN, aux=None, operand=True) -> Prepared:
    """Hadamard-256 rotation + per-row quantization (reference `prepare*` family)."""
    _need_cuda(x, aux)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("unsupported rotated integer operand")
    rows, width = x.shape
    stride = stride_for(width, bits) if stride is None else stride
    words = stride // (32 // bits)
    storage = torch.empty(rows * (words + 1), dtype=torch.int32, device=x.device)
    op = torch.empty((rows, width), dtype=torch.int8, device=x.device) if (operand and bits == 4) else None
    norm = torch.empty((rows, width), dtype=torch.bfloat16, device=x.device) if kind == PREP_NORM_STORE else None
    aux_ld = aux.stride(0) if (aux is not None and aux.dim() == 2) else 0
    if x.stride(1) != 1 or (aux is not None and aux.stride(-1) != 1):
        raise ValueError("packing inputs must have contiguous rows")
    _call("clefq_prepare", _stream(), kind, bits, _ptr(x), x.stride(0), _ptr(aux), aux_ld, rows, width, stride,
          _ptr(storage), _ptr(op), width if op is not None else 0, _ptr(norm), width)
    codes = storage[: rows * words].view(rows, words)
    scales = storage[rows * words:].view(torch.float32)
    return Prepared(storage, codes, scales, op, norm, bits, stride)


def retile_codes(codes, rows, cols, bits=4):
    """src/quantized.rs:542-572."""
    _need_cuda(codes)
    words = cols // (32 // bits)
    out = torch.empty(rows * words, dtype=torch.int32, device=codes.device)
    _call("clefq_retile", _stream(), _ptr(codes), rows, cols, bits, codes.shape[-1], _ptr(out))
    return out


@dataclass
class QuantizedWeight:
    """src/quantized.rs:12-20: tiled codes, compact f32 scales, shape, stride, bits."""
    codes: torch.Tensor
    scales: torch.Tensor
    rows: int
    cols: int
    stride: int
    bits: int


def load_quantized_weight(w, bits=4, tiled=False) -> QuantizedWeight:
    """src/quantized.rs:147-234 (after the precision policy, which `clefq.loading` holds): BF16
    [rows][cols] -> prepare (weights rotate and quantize like activations) -> retile, one
    clefq_load_weight call.  tiled=True: w holds the checkpoint's tiled256x64 byte order
    (src/checkpoint.rs:20-100) under its logical [rows][cols] shape."""
    _need_cuda(w)
    rows, cols = w.shape
    if rows % 256 or cols % 256:
        raise ValueError("unsupported quantized weight shape")
    w = w.contiguous()
    codes = torch.empty(rows * cols * bits // 32, dtype=torch.int32, device=w.device)
    scales = torch.empty(rows, dtype=torch.float32, device=w.device)
    need = lib().clefq_load_weight_workspace_size(rows, cols, bits, int(tiled))
    ws = torch.empty(need, dtype=torch.uint8, device=w.device)
    _call("clefq_load_weight", _stream(), _ptr(w), rows, cols, bits, int(tiled), _ptr(codes), _ptr(scales), _ptr(ws),
          need)
    return QuantizedWeight(codes, scales, rows, cols, stride_for(cols, bits), bits)


def untile_bf16(w):
    """Checkpoint tiled256x64 order -> row-major rows (src/checkpoint.rs:67-100), on the device."""
    _need_cuda(w)
    rows, cols = w.shape
    out = torch.empty_like(w)
    _call("clefq_untile_bf16", _stream(), _ptr(w.contiguous()), rows, cols, _ptr(out))
    return out


# ---------------------------------------------------------------------------------------
# Projections
# ---------------------------------------------------------------------------------------
def project_prepared(rows, w: QuantizedWeight, a: Prepared, residual=None, out_dtype=torch.bfloat16):
    """src/quantized.rs:470-537 (kernel h3_gemm_i{4,8}_256[_residual])."""
    if residual is not None and (residual.shape != (rows, w.rows) or residual.dtype != torch.bfloat16):
        raise ValueError("projection residual shape/dtype mismatch")
    dev = a.codes.device
    out = torch.empty((rows, w.rows), dtype=out_dtype, device=dev)
    odt = F32 if out_dtype == torch.float32 else BF16
    rld = residual.stride(0) if residual is not None else 0
    if a.operand is not None and a.bits == 4:
        _call("clefq_gemm_s8", _stream(), 4, _ptr(a.operand), a.operand.stride(0), _ptr(a.scales), rows,
              _ptr(w.codes), _ptr(w.scales), w.rows, w.cols, _ptr(residual), rld, odt, _ptr(out), w.rows)
    else:
        ws_bytes = lib().clefq_gemm_workspace_size(rows, w.cols, a.bits)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        _call("clefq_gemm", _stream(), a.bits, _ptr(a.codes), a.codes.shape[1], _ptr(a.scales), rows, _ptr(w.codes),
              _ptr(w.scales), w.rows, w.cols, _ptr(residual), rld, odt, _ptr(out), w.rows, _ptr(ws), ws_bytes)
    return out


def project_quantized(x, w: QuantizedWeight, residual=None, out_dtype=torch.bfloat16):
    """src/quantized.rs:235-251."""
    if x.shape[1] != w.cols or x.dtype != torch.bfloat16:
        raise ValueError("quantized projection shape/dtype mismatch")
    a = prepare(x, w.bits, w.stride)
    return project_prepared(x.shape[0], w, a, residual, out_dtype)


def swiglu(gate, up):
    """src/ops.rs:9-29."""
    _need_cuda(gate, up)
    if gate.shape != up.shape or gate.dtype != torch.bfloat16 or up.dtype != torch.bfloat16:
        raise ValueError("SwiGLU shape/dtype mismatch")
    gate, up = gate.contiguous(), up.contiguous()
    out = torch.empty_like(gate)
    _call("clefq_swiglu", _stream(), _ptr(gate), _ptr(up), gate.numel(), _ptr(out))
    return out


def silu(x):
    """bf16(x / (1 + exp(-x))) of BF16 values, as the SwiGLU GEMM epilogue computes it
    (clefq_silu)."""
    _need_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError("SiLU takes BF16")
    x = x.contiguous()
    out = torch.empty_like(x)
    _call("clefq_silu", _stream(), _ptr(x), x.numel(), _ptr(out))
    return out


def project_swiglu(gate, up, w: QuantizedWeight, residual=None):
    """src/quantized.rs:406-439: fused SwiGLU packing then the projection."""
    if gate.shape != up.shape or gate.shape[1] != w.cols:
        raise ValueError("SwiGLU projection width mismatch")
    a = prepare(gate, w.bits, w.stride, PREP_SWIGLU, up)
    return project_prepared(gate.shape[0], w, a, residual)


def mlp(x, gate: QuantizedWeight, up: QuantizedWeight, down: QuantizedWeight, residual=None, workspace=None):
    """Dense INT4 SwiGLU MLP block (src/backbone.rs:880-894 + src/quantized.rs:406-439),
    one C-ABI call: prepare -> gate|up -> fused SwiGLU packing -> down (+ residual).
    A host (CPU) x runs through `mlp_host` and returns a host tensor."""
    if not x.is_cuda:
        return mlp_host(x, gate, up, down, residual=residual, workspace=workspace)
    m, hidden = x.shape
    inter = gate.rows
    if not (gate.cols == up.cols == hidden and up.rows == inter and down.cols == inter and down.rows == hidden):
        raise ValueError("MLP weight shapes do not chain")
    out = torch.empty((m, hidden), dtype=torch.bfloat16, device=x.device)
    need = lib().clefq_mlp_workspace_size(m, hidden, inter)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    _call("clefq_mlp", _stream(), _ptr(x), m, hidden, inter, _ptr(gate.codes), _ptr(gate.scales), _ptr(up.codes),
          _ptr(up.scales), _ptr(down.codes), _ptr(down.scales), _ptr(residual), _ptr(out), _ptr(workspace), need)
    return out


def normalized_mlp(x, norm_weight, gate: QuantizedWeight, up: QuantizedWeight, down: QuantizedWeight, out=None,
                   workspace=None):
    """Pre-norm MLP block with x as its residual (src/quantized.rs:348-404), one C-ABI call:
    RMSNorm fused into the packing of x -> gate|up -> SwiGLU packing -> down + x.
    norm_weight: BF16 [hidden] (applied as weight + 1, eps 1e-6).  out may be x."""
    _need_cuda(x, norm_weight)
    m, hidden = x.shape
    inter = gate.rows
    if not (gate.cols == up.cols == hidden and up.rows == inter and down.cols == inter and down.rows == hidden):
        raise ValueError("MLP weight shapes do not chain")
    if norm_weight.shape != (hidden,) or norm_weight.dtype != torch.bfloat16 or x.dtype != torch.bfloat16:
        raise ValueError("normalized MLP shape/dtype mismatch")
    if out is None:
        out = torch.empty((m, hidden), dtype=torch.bfloat16, device=x.device)
    need = lib().clefq_mlp_workspace_size(m, hidden, inter)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    _call("clefq_normalized_mlp", _stream(), _ptr(x), m, hidden, inter, _ptr(norm_weight.contiguous()),
          _ptr(gate.codes), _ptr(gate.scales), _ptr(up.codes), _ptr(up.scales), _ptr(down.codes), _ptr(down.scales),
          _ptr(out), _ptr(workspace), need)
    return out


def project_pair_prepared(rows, w0: QuantizedWeight, w1: QuantizedWeight, a: Prepared, out=None):
    """Two projections of one prepared input in one launch (gate and up of an MLP):
    returns BF16 [rows][2n] = [x.w0 | x.w1] (clefq_gemm_pair_s8)."""
    if a.operand is None or a.bits != 4 or w0.rows != w1.rows or w0.cols != w1.cols:
        raise ValueError("paired projection needs an int4 s8 operand and two weights of one shape")
    n = w0.rows
    if out is None:
        out = torch.empty((rows, 2 * n), dtype=torch.bfloat16, device=a.codes.device)
    _call("clefq_gemm_pair_s8", _stream(), _ptr(a.operand), a.operand.stride(0), _ptr(a.scales), rows,
          _ptr(w0.codes), _ptr(w0.scales), _ptr(w1.codes), _ptr(w1.scales), n, w0.cols, _ptr(out), out.stride(0))
    return out


def project_swiglu_prepared(rows, gate: QuantizedWeight, up: QuantizedWeight, a: Prepared, out=None):
    """Gate and up projections of one prepared input with SwiGLU in the GEMM epilogue, the
    gate|up step of the MLP block: returns BF16 [rows][n] = swiglu(x.gate, x.up)
    (clefq_gemm_swiglu_s8)."""
    if a.operand is None or a.bits != 4 or gate.rows != up.rows or gate.cols != up.cols:
        raise ValueError("SwiGLU projection needs an int4 s8 operand and two weights of one shape")
    n = gate.rows
    if out is None:
        out = torch.empty((rows, n), dtype=torch.bfloat16, device=a.codes.device)
    _call("clefq_gemm_swiglu_s8", _stream(), _ptr(a.operand), a.operand.stride(0), _ptr(a.scales), rows,
          _ptr(gate.codes), _ptr(gate.scales), _ptr(up.codes), _ptr(up.scales), n, gate.cols, _ptr(out),
          out.stride(0))
    return out


HOST_STREAMING = 1


def mlp_host(x, gate: QuantizedWeight, up: QuantizedWeight, down: QuantizedWeight, residual=None, out=None,
             chunk_rows=1024, workspace=None, sync=True, streaming=False, done_event=None):
    """The MLP block from host rows to host rows (clefq_mlp_host): row chunks stream through
    the GPU with their PCIe copies overlapping the neighbouring chunks' kernels.  x, residual
    and out are CPU bf16 [m][hidden] (pinned memory for overlap).  With sync=False the call
    returns once enqueued; out is ready when the current stream reaches it, or when
    done_event (a torch.cuda.Event) fires if one is given.  streaming=True lets the input
    copies start before earlier work on the stream ends, so back-to-back calls overlap (the
    workspace must then serve only these calls)."""
    if x.is_cuda or (residual is not None and residual.is_cuda):
        raise ValueError("mlp_host takes host tensors")
    m, hidden = x.shape
    inter = gate.rows
    if not (gate.cols == up.cols == hidden and up.rows == inter and down.cols == inter and down.rows == hidden):
        raise ValueError("MLP weight shapes do not chain")
    x = x.contiguous()
    if residual is not None:
        residual = residual.contiguous()
    if out is None:
        out = torch.empty((m, hidden), dtype=torch.bfloat16, pin_memory=x.is_pinned())
    chunk_rows = max(1, min(int(chunk_rows), m))
    need = lib().clefq_mlp_host_workspace_size(chunk_rows, hidden, inter, int(residual is not None))
    if need < 0:
        raise ValueError("unsupported MLP shape")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=gate.codes.device)
    ev = None
    if done_event is not None:
        if not done_event.cuda_event:
            done_event.record()  # torch creates the CUDA event at its first record
        ev = ctypes.c_void_p(done_event.cuda_event)
    _call("clefq_mlp_host", _stream(), _ptr(x), m, hidden, inter, _ptr(gate.codes), _ptr(gate.scales), _ptr(up.codes),
          _ptr(up.scales), _ptr(down.codes), _ptr(down.scales), _ptr(residual), _ptr(out), chunk_rows,
          HOST_STREAMING if streaming else 0, ev, _ptr(workspace), need)
    if sync:
        if done_event is not None:
            done_event.synchronize()
        torch.cuda.current_stream().synchronize()
    return out


# ---------------------------------------------------------------------------------------
# Omni MoE operators (src/omni.rs)
# ---------------------------------------------------------------------------------------
def omni_route(logits, topk=TOP_K):
    """src/omni.rs:170-190 -> routes f32 [tokens][2*topk]."""
    _need_cuda(logits)
    tokens, experts = logits.shape
    if not (0 < topk <= experts <= 128):
        raise ValueError("invalid expert router shape")
    dt = F32 if logits.dtype == torch.float32 else BF16
    logits = logits.contiguous()
    out = torch.empty((tokens, 2 * topk), dtype=torch.float32, device=logits.device)
    _call("clefq_route", _stream(), _ptr(logits), dt, tokens, experts, topk, _ptr(out))
    return out


def omni_route_linear(x, router_weight, topk=TOP_K, logits_out=False):
    """Router linear (BF16 projection by mlp.gate) and omni_route in one kernel
    (src/omni.rs:760-765) -> routes f32 [tokens][2*topk], and the BF16 logits if asked."""
    _need_cuda(x, router_weight)
    if x.dtype != torch.bfloat16 or router_weight.dtype != torch.bfloat16 or x.dim() != 2 or \
            router_weight.dim() != 2 or x.shape[1] != router_weight.shape[1]:
        raise ValueError("router linear shape/dtype mismatch")
    tokens, hidden = x.shape
    experts = router_weight.shape[0]
    x, router_weight = x.contiguous(), router_weight.contiguous()
    routes = torch.empty((tokens, 2 * topk), dtype=torch.float32, device=x.device)
    logits = torch.empty((tokens, experts), dtype=torch.bfloat16, device=x.device) if logits_out else None
    _call("clefq_route_linear", _stream(), _ptr(x), _ptr(router_weight), tokens, hidden, experts, topk, _ptr(routes),
          _ptr(logits))
    return (routes, logits) if logits_out else routes


def omni_group_routes_ordered(routes, experts=EXPERTS):
    """src/omni.rs:213-245 -> (groups f32 [experts][tokens+1], order f32 [tokens][topk])."""
    tokens, width = routes.shape
    topk = width // 2
    groups = torch.zeros((experts, tokens + 1), dtype=torch.float32, device=routes.device)
    order = torch.zeros((tokens, topk), dtype=torch.float32, device=routes.device)
    need = lib().clefq_group_workspace_size(tokens, topk, experts)
    ws = torch.empty(need, dtype=torch.uint8, device=routes.device)
    _call("clefq_group_routes", _stream(), _ptr(routes), tokens, topk, experts, _ptr(groups), _ptr(order), _ptr(ws),
          need)
    return groups, order


def omni_group_routes(routes, experts=EXPERTS):
    """src/omni.rs:192-212."""
    return omni_group_routes_ordered(routes, experts)[0]


def omni_expert_tasks(groups, tokens, topk=TOP_K):
    """src/omni.rs:126-169 task list (reference format)."""
    experts = groups.shape[0]
    n = 1 + 2 * (-(-tokens * topk // 16) + experts - 1)
    tasks = torch.zeros(n, dtype=torch.float32, device=groups.device)
    _call("clefq_expert_tasks", _stream(), _ptr(groups), tokens, experts, _ptr(tasks))
    return tasks


def omni_compact_routes(routes, experts=EXPERTS):
    """src/omni.rs:126-169 -> (combined buffer groups||order||tasks, order)."""
    tokens = routes.shape[0]
    groups, order = omni_group_routes_ordered(routes, experts)
    tasks = omni_expert_tasks(groups, tokens, routes.shape[1] // 2)
    return torch.cat([groups.reshape(-1), order.reshape(-1), tasks]), order


def omni_expert(x_prepared: Prepared, routes, groups, w: QuantizedWeight, input_routed: bool, experts=EXPERTS):
    """src/omni.rs:289-534 grouped INT4 experts: out[route][c] BF16 [tokens*topk][n]."""
    tokens, width = routes.shape
    topk = width // 2
    n = w.rows // experts
    k = w.cols
    out = torch.empty((tokens * topk, n), dtype=torch.bfloat16, device=routes.device)
    need = lib().clefq_expert_workspace_size(tokens, topk, experts, k)
    ws = torch.empty(need, dtype=torch.uint8, device=routes.device)
    _call("clefq_expert", _stream(), _ptr(x_prepared.codes), x_prepared.codes.shape[1], _ptr(x_prepared.scales),
          _ptr(w.codes), _ptr(w.scales), _ptr(groups), tokens, topk, experts, k, n, int(input_routed), _ptr(out),
          _ptr(ws), need)
    return out


def omni_gate_up(x_prepared: Prepared, routes, groups, gate: QuantizedWeight, up: QuantizedWeight,
                 experts=EXPERTS):
    """src/omni.rs:302-373 fused gate/up experts: hidden[route] = bf16(bf16(silu(g)) * u),
    SwiGLU in the GEMM epilogue -> BF16 [tokens*topk][n] in route order."""
    tokens, width = routes.shape
    topk = width // 2
    n = gate.rows // experts
    k = gate.cols
    if up.rows != gate.rows or up.cols != k:
        raise ValueError("gate and up expert weights differ in shape")
    out = torch.empty((tokens * topk, n), dtype=torch.bfloat16, device=routes.device)
    need = lib().clefq_expert_workspace_size(tokens, topk, experts, k)
    ws = torch.empty(need, dtype=torch.uint8, device=routes.device)
    _call("clefq_expert_gate_up", _stream(), _ptr(x_prepared.codes), x_prepared.codes.shape[1],
          _ptr(x_prepared.scales), _ptr(gate.codes), _ptr(gate.scales), _ptr(up.codes), _ptr(up.scales), _ptr(groups),
          tokens, topk, experts, k, n, _ptr(out), _ptr(ws), need)
    return out


def omni_combine_ordered(values, routes, order):
    """src/omni.rs:246-278."""
    tokens, width2 = routes.shape
    topk = width2 // 2
    if values.shape[0] != tokens * topk or values.shape[1] % 8 or values.dtype != torch.bfloat16:
        raise ValueError("unsupported ordered Omni accumulation")
    out = torch.empty((tokens, values.shape[1]), dtype=torch.bfloat16, device=values.device)
    _call("clefq_combine", _stream(), _ptr(values), _ptr(routes), _ptr(order), tokens, topk, values.shape[1],
          _ptr(out))
    return out


def omni_combine(values, routes):
    """src/omni.rs:535-556 (ascending order found per token)."""
    return omni_combine_ordered(values, routes, None)


def omni_moe(x, logits, gate: QuantizedWeight, up: QuantizedWeight, down: QuantizedWeight, experts=EXPERTS,
             topk=TOP_K, workspace=None, routes_out=None, router_weight=None, out=None):
    """The MoE block of forward_layers_cached (src/omni.rs:761-857), one C-ABI call.  Pass
    router_weight (BF16 [experts][hidden]) instead of logits to fuse the router linear in."""
    tokens, hidden = x.shape
    inter = gate.rows // experts
    if out is None:
        out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=x.device)
    need = lib().clefq_moe_workspace_size(tokens, hidden, inter, experts, topk)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    if router_weight is not None:
        if logits is not None or router_weight.shape != (experts, hidden):
            raise ValueError("pass either logits or a router weight [experts][hidden]")
        logits, dt = router_weight.contiguous(), ROUTER_WEIGHT_BF16
    else:
        dt = F32 if logits.dtype == torch.float32 else BF16
    _call("clefq_moe", _stream(), _ptr(x), _ptr(logits), dt, tokens, hidden, inter, experts, topk, _ptr(gate.codes),
          _ptr(gate.scales), _ptr(up.codes), _ptr(up.scales), _ptr(down.codes), _ptr(down.scales), _ptr(out),
          _ptr(routes_out), _ptr(workspace), need)
    return out
