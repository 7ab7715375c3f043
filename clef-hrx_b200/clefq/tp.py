"""Tensor-parallel dense INT4 SwiGLU MLP block over torch.distributed (one process per GPU).

The reference runs the MLP block (src/backbone.rs:880-894, src/quantized.rs:406-439) on one
GPU.  Here the intermediate dimension I is split over G ranks: rank r owns gate/up rows
[r*I/G, (r+1)*I/G) and down rows [r*H/G, (r+1)*H/G).  Every rank holds the whole input:

    pack x -> gate|up of the rank's rows -> SwiGLU shard row maxima -> all-reduce(MAX)
    -> pack the shard with the full-row maxima (same scales on every rank) -> all-gather the
    int4 code shards -> full s8 operand -> down of the rank's output rows (+ residual columns)
    -> all-gather the output columns -> [M][H]

Hadamard groups never straddle a shard, the row scale comes from the whole row and every
output column of down sees the full K, so the output equals `clefq.mlp` bit for bit.  The
exchanged bytes per block are M*I/2 (packed codes), M*H*2 (output) and M*4 (maxima).

`mlp_tp` runs these steps as separate kernels and torch.distributed collectives (any
backend; the CPU tests drive it over gloo).  `mlp_tp_fused` is the B200 path: one C-ABI call
(clefq_tp_mlp) over a `TpComm`, whose packing kernel and GEMM epilogue store their shards
straight into every rank's symmetric buffer over NVLink, ordered by device barriers.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .comm import Comm, all_gather_rows as _all_gather


@dataclass
class MlpShard:
    """This rank's slices of the MLP weights (QuantizedWeight each, or oracle tuples in tests)."""
    gate: object
    up: object
    down: object
    rank: int
    world: int
    hidden: int
    inter: int


def shard_mlp(gate, up, down, rank: int, world: int) -> MlpShard:
    """Cuts rank `rank`'s rows out of the tiled weights (tiles are ordered by 128-row block,
    so a row range that is a multiple of 128 is one contiguous slice)."""
    from . import QuantizedWeight
    inter, hidden = gate.rows, down.rows
    if inter % (256 * world) or hidden % (128 * world):
        raise ValueError("intermediate must split into whole 256-groups and hidden into 128-row tiles")

    def cut(w, per):
        words_per_row = w.codes.numel() // w.rows
        lo, hi = rank * per, (rank + 1) * per
        return QuantizedWeight(w.codes[lo * words_per_row:hi * words_per_row], w.scales[lo:hi], per, w.cols,
                               w.stride, w.bits)
    return MlpShard(cut(gate, inter // world), cut(up, inter // world), cut(down, hidden // world), rank, world,
                    hidden, inter)


class CudaTpOps:
    """The device steps, each one libclefq.so entry point."""

    def __init__(self):
        from . import lib
        lib()  # raises when the library has not been built: there is no fallback

    def pack_x(self, x):
        from . import prepare, stride_for
        return prepare(x, 4, stride_for(x.shape[1]))

    def gate_up(self, xq, m, shard):
        from . import _call, _stream, _ptr
        n = shard.gate.rows
        gu = torch.empty(m, 2 * n, dtype=torch.bfloat16, device=xq.codes.device)
        for i, w in enumerate((shard.gate, shard.up)):
            _call("clefq_gemm_s8", _stream(), 4, _ptr(xq.operand), xq.operand.stride(0), _ptr(xq.scales), m,
                  _ptr(w.codes), _ptr(w.scales), n, w.cols, None, 0, 0, gu.data_ptr() + i * n * 2, 2 * n)
        return gu

    def rowmax(self, gu):
        from . import _call, _stream, _ptr, PREP_SWIGLU
        m, n2 = gu.shape
        n = n2 // 2
        mx = torch.empty(m, dtype=torch.float32, device=gu.device)
        _call("clefq_prepare_rowmax", _stream(), PREP_SWIGLU, _ptr(gu), n2, gu.data_ptr() + n * 2, n2, m, n, _ptr(mx))
        return mx

    def pack_hidden(self, gu, rowmax):
        """int4 codes [m][n/8] (int32) and f32 scales [m] of the SwiGLU shard."""
        from . import _call, _stream, _ptr, PREP_SWIGLU
        m, n2 = gu.shape
        n = n2 // 2
        words = n // 8
        storage = torch.empty(m * (words + 1), dtype=torch.int32, device=gu.device)
        operand = torch.empty(m, n, dtype=torch.int8, device=gu.device)  # selects the table kernel
        _call("clefq_prepare_scaled", _stream(), PREP_SWIGLU, 4, _ptr(gu), n2, gu.data_ptr() + n * 2, n2, m, n, n,
              _ptr(rowmax), _ptr(storage), _ptr(operand), n)
        return storage[:m * words].view(m, words), storage[m * words:].view(torch.float32)

    def gather_unpack(self, codes_all, inter):
        from . import _call, _stream, _ptr
        world, m, words = codes_all.shape
        op = torch.empty(m, inter, dtype=torch.int8, device=codes_all.device)
        _call("clefq_tp_gather_unpack", _stream(), _ptr(codes_all), world, m, words * 8, _ptr(op), inter)
        return op

    def down(self, operand, scales, shard, residual):
        from . import _call, _stream, _ptr
        m = operand.shape[0]
        w = shard.down
        out = torch.empty(m, w.rows, dtype=torch.bfloat16, device=operand.device)
        res, rld = None, 0
        if residual is not None:
            res = residual.data_ptr() + shard.rank * w.rows * 2
            rld = residual.stride(0)
        _call("clefq_gemm_s8", _stream(), 4, _ptr(operand), operand.stride(0), _ptr(scales), m, _ptr(w.codes),
              _ptr(w.scales), w.rows, w.cols, res, rld, 0, _ptr(out), w.rows)
        return out

    def interleave(self, out_all):
        from . import _call, _stream, _ptr
        world, m, hs = out_all.shape
        out = torch.empty(m, world * hs, dtype=out_all.dtype, device=out_all.device)
        esz = out_all.element_size()
        _call("clefq_tp_interleave", _stream(), _ptr(out_all), world, m, hs * esz, _ptr(out), world * hs * esz)
        return out


def mlp_tp(x: torch.Tensor, shard: MlpShard, residual=None, group=None, ops=None) -> torch.Tensor:
    """Tensor-parallel MLP block; every rank passes the same x (and residual) and gets the
    whole output [M][H]."""
    ops = ops if ops is not None else CudaTpOps()
    world = dist.get_world_size(group)
    if shard.world != world:
        raise ValueError("MLP shard does not match the process group size")
    m = x.shape[0]
    xq = ops.pack_x(x)
    gu = ops.gate_up(xq, m, shard)
    mx = ops.rowmax(gu)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
    codes, scales = ops.pack_hidden(gu, mx)
    codes_all = torch.empty((world,) + tuple(codes.shape), dtype=codes.dtype, device=codes.device)
    _all_gather(codes_all, codes, group)
    operand = ops.gather_unpack(codes_all, shard.inter)
    part = ops.down(operand, scales, shard, residual)
    out_all = torch.empty((world,) + tuple(part.shape), dtype=part.dtype, device=part.device)
    _all_gather(out_all, part, group)
    return ops.interleave(out_all)


TpComm = Comm  # the communicator of the fused path (clefq.comm)


def tp_mlp_region_bytes(m: int, hidden: int, inter: int, world: int) -> int:
    from . import lib
    n = lib().clefq_tp_mlp_region_bytes(m, hidden, inter, world)
    if n < 0:
        raise ValueError("unsupported tensor-parallel MLP shape")
    return n


def mlp_tp_fused(x: torch.Tensor, shard: MlpShard, comm: TpComm, residual=None, workspace=None, out=None):
    """Tensor-parallel MLP block in one C-ABI call (clefq_tp_mlp); every rank passes the same
    x (and residual) and gets the whole output [M][H], bit-identical to `clefq.mlp`."""
    from . import _call, _need_cuda, _ptr, _stream, lib
    _need_cuda(x, residual)
    if shard.world != comm.world or shard.rank != comm.rank:
        raise ValueError("MLP shard does not match the communicator")
    m, hidden = x.shape
    if hidden != shard.hidden:
        raise ValueError("MLP input width does not match the shard")
    x = x.contiguous()
    if residual is not None:
        residual = residual.contiguous()
        if residual.shape != x.shape:
            raise ValueError("residual shape must match x")
    need = lib().clefq_tp_mlp_workspace_size(m, hidden, shard.inter, shard.world)
    if need < 0:
        raise ValueError("unsupported tensor-parallel MLP shape")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty((m, hidden), dtype=torch.bfloat16, device=x.device)
    g, u, d = shard.gate, shard.up, shard.down
    _call("clefq_tp_mlp", comm.handle, _stream(), _ptr(x), m, hidden, shard.inter, _ptr(g.codes), _ptr(g.scales),
          _ptr(u.codes), _ptr(u.scales), _ptr(d.codes), _ptr(d.scales), _ptr(residual), _ptr(out), _ptr(workspace),
          need)
    return out
