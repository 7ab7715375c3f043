"""Expert-parallel Omni MoE layer over torch.distributed (one process per GPU).

The reference runs the MoE block on one GPU (src/omni.rs:761-857).  Here the experts are
split into contiguous id ranges, rank r owning [r * E/G, (r + 1) * E/G), and every rank
keeps its own tokens:

    route (local) -> pack each token once (int4 codes + scale) -> plan + pack one record
    per route, grouped by destination -> all-to-all -> grouped expert FFN on the received
    records, each output weighted by its probability -> all-to-all back -> the
    reference's ascending-expert BF16 chain on the home rank

The result is bit-identical to `clefq.omni_moe` on one GPU (see ep.cu).  The collectives
are `all_to_all_single` on NCCL; on backends without all-to-all (gloo, for host tests)
the same exchange runs as paired send/recv.  Record and product buffers are allocated per
call; the counts exchange is the one host synchronisation of the layer.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class ExpertShard:
    """This rank's experts: tiled int4 weights of experts [base, base + count) in the
    layout of `clefq.omni_moe` (gate/up [count*inter][hidden], down [count*hidden][inter])."""
    gate: object
    up: object
    down: object
    base: int
    count: int
    experts: int
    inter: int


def shard_experts(gate, up, down, experts: int, inter: int, hidden: int, rank: int, world: int) -> ExpertShard:
    """Slices the global tiled expert weights (QuantizedWeight) down to this rank's range.
    Tiles are ordered by 128-row block, so an expert range is a contiguous slice."""
    from . import QuantizedWeight
    if experts % world:
        raise ValueError("experts must divide evenly over ranks")
    per = experts // world
    base = rank * per

    def cut(w, rows_per_expert):
        words_per_row = w.codes.numel() // w.rows
        lo, hi = base * rows_per_expert, (base + per) * rows_per_expert
        return QuantizedWeight(w.codes[lo * words_per_row:hi * words_per_row], w.scales[lo:hi], hi - lo, w.cols,
                               w.stride, w.bits)
    return ExpertShard(cut(gate, inter), cut(up, inter), cut(down, hidden), base, per, experts, inter)


def _exchange(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group):
    """all_to_all_single(out, inp) with split sizes along dim 0."""
    if dist.get_backend(group) == "nccl":
        dist.all_to_all_single(out, inp, list(out_splits), list(in_splits), group=group)
        return
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    in_off = [0]
    for c in in_splits:
        in_off.append(in_off[-1] + c)
    out_off = [0]
    for c in out_splits:
        out_off.append(out_off[-1] + c)
    reqs = []
    for peer in range(world):
        if peer == rank:
            out[out_off[peer]:out_off[peer + 1]].copy_(inp[in_off[peer]:in_off[peer + 1]])
            continue
        if in_splits[peer]:
            reqs.append(dist.isend(inp[in_off[peer]:in_off[peer + 1]].contiguous(), dist.get_global_rank(group, peer)
                                   if group is not None else peer, group=group))
        if out_splits[peer]:
            reqs.append(dist.irecv(out[out_off[peer]:out_off[peer + 1]], dist.get_global_rank(group, peer)
                                   if group is not None else peer, group=group))
    for r in reqs:
        r.wait()


class CudaEpOps:
    """The device steps of the layer, each one libclefq.so entry point."""

    def __init__(self):
        from . import lib
        lib()  # raises when the library has not been built: there is no fallback

    def route(self, logits, topk):
        from . import omni_route
        return omni_route(logits, topk)

    def pack_tokens(self, x):
        from . import prepare, stride_for
        p = prepare(x, 4, stride_for(x.shape[1]), operand=False)
        return p.codes, p.scales

    def plan(self, routes, topk, experts, world):
        from . import _call, _stream, _ptr, lib
        tokens = routes.shape[0]
        counts = torch.empty(world, dtype=torch.int64, device=routes.device)
        slots = torch.empty(max(tokens * topk, 1), dtype=torch.int32, device=routes.device)
        need = lib().clefq_moe_ep_plan_workspace_size(world)
        ws = torch.empty(need, dtype=torch.uint8, device=routes.device)
        _call("clefq_moe_ep_plan", _stream(), _ptr(routes), tokens, topk, experts, world, _ptr(counts), _ptr(slots),
              _ptr(ws), need)
        return counts, slots

    def record_bytes(self, hidden):
        from . import lib
        return lib().clefq_moe_ep_record_bytes(hidden)

    def pack_records(self, codes, scales, routes, topk, slots, n_send, hidden):
        from . import _call, _stream, _ptr
        rec = self.record_bytes(hidden)
        send = torch.empty(max(n_send, 1) * rec, dtype=torch.uint8, device=codes.device)
        _call("clefq_moe_ep_pack", _stream(), _ptr(codes), codes.shape[1], _ptr(scales), codes.shape[0], hidden,
              _ptr(routes), topk, _ptr(slots), _ptr(send))
        return send

    def experts(self, records, n, hidden, shard: ExpertShard):
        from . import _call, _stream, _ptr, lib
        products = torch.empty(max(n, 1), hidden, dtype=torch.bfloat16, device=records.device)
        need = lib().clefq_moe_ep_experts_workspace_size(n, hidden, shard.inter, shard.count)
        ws = torch.empty(need, dtype=torch.uint8, device=records.device)
        _call("clefq_moe_ep_experts", _stream(), _ptr(records), n, hidden, shard.inter, shard.base, shard.count,
              _ptr(shard.gate.codes), _ptr(shard.gate.scales), _ptr(shard.up.codes), _ptr(shard.up.scales),
              _ptr(shard.down.codes), _ptr(shard.down.scales), _ptr(products), _ptr(ws), need)
        return products

    def combine(self, products, slots, routes, topk, hidden):
        from . import _call, _stream, _ptr
        tokens = routes.shape[0]
        out = torch.empty(tokens, hidden, dtype=torch.bfloat16, device=routes.device)
        _call("clefq_moe_ep_combine", _stream(), _ptr(products), _ptr(slots), _ptr(routes), tokens, topk, hidden,
              _ptr(out))
        return out


def omni_moe_ep(x: torch.Tensor, logits: torch.Tensor, shard: ExpertShard, topk: int = 8, group=None, ops=None):
    """Expert-parallel Omni MoE block for this rank's tokens; returns (out, routes)."""
    ops = ops if ops is not None else CudaEpOps()
    world = dist.get_world_size(group)
    tokens, hidden = x.shape
    if shard.count * world != shard.experts:
        raise ValueError("expert shard does not match the process group size")
    routes = ops.route(logits, topk)
    codes, scales = ops.pack_tokens(x)
    send_counts, slots = ops.plan(routes, topk, shard.experts, world)
    recv_counts = torch.empty_like(send_counts)
    _exchange(recv_counts, send_counts, [1] * world, [1] * world, group)
    sc = [int(c) for c in send_counts.tolist()]
    rc = [int(c) for c in recv_counts.tolist()]
    n_send, n_recv = sum(sc), sum(rc)
    rec = ops.record_bytes(hidden)
    send = ops.pack_records(codes, scales, routes, topk, slots, n_send, hidden)
    recv = torch.empty(max(n_recv, 1) * rec, dtype=torch.uint8, device=send.device)
    _exchange(recv, send, [c * rec for c in rc], [c * rec for c in sc], group)
    products = ops.experts(recv, n_recv, hidden, shard)
    back = torch.empty(max(n_send, 1), hidden, dtype=torch.bfloat16, device=products.device)
    _exchange(back, products, sc, rc, group)
    return ops.combine(back, slots, routes, topk, hidden), routes


def ep_layer_region_bytes(tokens: int, hidden: int, topk: int, world: int, recv_cap: int) -> int:
    from . import lib
    n = lib().clefq_moe_ep_layer_region_bytes(tokens, hidden, topk, world, recv_cap)
    if n < 0:
        raise ValueError("unsupported expert-parallel MoE layer shape")
    return n


def omni_moe_ep_fused(x: torch.Tensor, logits: torch.Tensor, shard: ExpertShard, comm, topk: int = 8,
                      recv_cap: int | None = None, workspace=None, out=None, router_weight=None):
    """Expert-parallel Omni MoE block in one C-ABI call (clefq_moe_ep_layer) over a
    `clefq.comm.Comm`: records and products are stored straight into the other ranks'
    symmetric buffers by the dispatch kernel and the expert down-GEMM epilogue, with no host
    synchronisation.  recv_cap (the same on every rank) defaults to world * tokens * topk, which
    always suffices when every rank has `tokens` tokens.  Pass router_weight (BF16 [experts]
    [hidden]) with logits=None to fuse the router linear in.  Returns (out, routes)."""
    from . import BF16, F32, ROUTER_WEIGHT_BF16, _call, _need_cuda, _ptr, _stream, lib
    if router_weight is not None:
        if logits is not None:
            raise ValueError("pass either logits or a router weight")
        logits = router_weight
    _need_cuda(x, logits)
    tokens, hidden = x.shape
    world = comm.world
    if shard.count * world != shard.experts or shard.base != comm.rank * shard.count:
        raise ValueError("expert shard does not match the communicator")
    if recv_cap is None:
        recv_cap = world * tokens * topk
    x = x.contiguous()
    logits = logits.contiguous()
    dt = ROUTER_WEIGHT_BF16 if router_weight is not None else (F32 if logits.dtype == torch.float32 else BF16)
    need = lib().clefq_moe_ep_layer_workspace_size(tokens, hidden, shard.inter, shard.experts, topk, world, recv_cap)
    if need < 0:
        raise ValueError("unsupported expert-parallel MoE layer shape")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    if out is None:
        out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=x.device)
    routes = torch.empty((tokens, 2 * topk), dtype=torch.float32, device=x.device)
    _call("clefq_moe_ep_layer", comm.handle, _stream(), _ptr(x), _ptr(logits), dt, tokens, hidden, shard.inter,
          shard.experts, topk, recv_cap, _ptr(shard.gate.codes), _ptr(shard.gate.scales), _ptr(shard.up.codes),
          _ptr(shard.up.scales), _ptr(shard.down.codes), _ptr(shard.down.scales), _ptr(out), _ptr(routes),
          _ptr(workspace), need)
    return out, routes
