"""Tensor-parallel dense MLP: the output equals the single-GPU block bit for bit.

- CPU, 2 gloo ranks: the real host orchestration (clefq.tp.mlp_tp) with oracle/numpy
  stand-ins for the device steps, against the oracle's mlp_block.
- GPU: the split packing entry points against clefq_prepare; G = 2 and 4 ranks simulated in
  one process (all-reduce and all-gathers done by hand) through every entry point, against
  clefq.mlp; 2 processes over NCCL (needs two GPUs).
"""
import ctypes
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


# ---------------------------------------------------------------------------------------
# CPU: 2 gloo ranks
# ---------------------------------------------------------------------------------------
T_M, T_H, T_I = 33, 512, 1024


def _cpu_problem():
    from oracle import oracle as o
    rng = np.random.default_rng(3)
    x = o.f32_to_bf16(rng.standard_normal((T_M, T_H)).astype(np.float32))
    x[5, 17] = 0x7FC0    # a NaN row: zero codes, infinite scale, as on one GPU
    gate = o.pack_weight(o.f32_to_bf16(rng.standard_normal((T_I, T_H)).astype(np.float32) * 0.05))
    up = o.pack_weight(o.f32_to_bf16(rng.standard_normal((T_I, T_H)).astype(np.float32) * 0.05))
    down = o.pack_weight(o.f32_to_bf16(rng.standard_normal((T_H, T_I)).astype(np.float32) * 0.05))
    return x, gate, up, down


def _cpu_worker(rank, world, port):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    from oracle import oracle as o
    from clefq.tp import MlpShard, mlp_tp
    from tests.tp_oracle_ops import OracleTpOps
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x, gate, up, down = _cpu_problem()

        def cut(w, rows, cols):
            per = rows // world
            words = cols // 8
            return (w[0][rank * per * words:(rank + 1) * per * words], w[1][rank * per:(rank + 1) * per])
        shard = MlpShard(cut(gate, T_I, T_H), cut(up, T_I, T_H), cut(down, T_H, T_I), rank, world, T_H, T_I)
        xt = torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16)
        out = mlp_tp(xt, shard, ops=OracleTpOps())
        ref = o.mlp_block(x, (gate[0], gate[1], T_I), (up[0], up[1], T_I), (down[0], down[1], T_H))
        got = out.view(torch.int16).numpy().view(np.uint16)
        bad = np.count_nonzero(got != ref)
        assert bad == 0, f"rank {rank}: {bad} mismatches"
    finally:
        dist.destroy_process_group()


def test_tp_host_logic_two_gloo_ranks():
    mp.start_processes(_cpu_worker, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")


def test_tp_host_logic_four_gloo_ranks():
    """Four ranks: one 256-group of the intermediate and 128 output columns per rank."""
    mp.start_processes(_cpu_worker, args=(4, _free_port()), nprocs=4, join=True, start_method="spawn")


# ---------------------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cq():
    import clefq
    clefq.lib()
    return clefq


def _weights(cq, hidden, inter, seed):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)

    def w(rows, cols):
        return cq.load_quantized_weight((torch.randn(rows, cols, device="cuda", generator=gen) * 0.05)
                                        .to(torch.bfloat16))
    return w(inter, hidden), w(inter, hidden), w(hidden, inter)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,width", [(7, 768), (300, 4096), (1000, 3072)])
def test_split_packing_matches_prepare(cq, rows, width):
    """rowmax + scaled packing of a whole row == clefq_prepare (codes, scales, operand)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(rows)
    gu = (torch.randn(rows, 2 * width, device="cuda", generator=gen) * 2).to(torch.bfloat16)
    gu[3 % rows, 5] = float("nan")
    from clefq.tp import CudaTpOps
    ops = CudaTpOps()
    ref = cq.prepare(gu[:, :width], 4, width, cq.PREP_SWIGLU, gu[:, width:])
    mx = ops.rowmax(gu)
    codes, scales = ops.pack_hidden(gu, mx)
    assert torch.equal(codes, ref.codes)
    assert torch.equal(scales.view(torch.int32), ref.scales.view(torch.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("world,m,residual", [(2, 300, False), (4, 129, True), (2, 2048, True)])
def test_tp_simulated_ranks_match_single_gpu(cq, world, m, residual):
    from clefq.tp import CudaTpOps, shard_mlp
    hidden, inter = 1024, 4096
    gate, up, down = _weights(cq, hidden, inter, 21)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(m)
    x = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16)
    res = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16) if residual else None
    shards = [shard_mlp(gate, up, down, r, world) for r in range(world)]
    ops = CudaTpOps()
    gus = [ops.gate_up(ops.pack_x(x), m, s) for s in shards]
    mx = torch.stack([ops.rowmax(g) for g in gus]).amax(dim=0)      # all-reduce(MAX)
    packed = [ops.pack_hidden(g, mx) for g in gus]
    for _, sc in packed[1:]:
        assert torch.equal(sc, packed[0][1])                           # same scales on every rank
    codes_all = torch.stack([c for c, _ in packed])                   # all-gather
    operand = ops.gather_unpack(codes_all, inter)
    parts = [ops.down(operand, packed[r][1], shards[r], res) for r in range(world)]
    out = ops.interleave(torch.stack(parts))                          # all-gather + interleave
    ref = cq.mlp(x, gate, up, down, residual=res)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (
        f"{(out.view(torch.int16) != ref.view(torch.int16)).sum().item()} mismatches")


def _nccl_worker(rank, world, port):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    import clefq as cq
    from clefq.tp import mlp_tp, shard_mlp
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        hidden, inter, m = 2048, 8192, 777
        gate, up, down = _weights(cq, hidden, inter, 9)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(5)                       # the same input on every rank
        x = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16)
        res = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16)
        out = mlp_tp(x, shard_mlp(gate, up, down, rank, world), residual=res)
        ref = cq.mlp(x, gate, up, down, residual=res)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_ranks_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_nccl_worker, args=(world, _free_port()), nprocs=world, join=True, start_method="spawn")


# ---------------------------------------------------------------------------------------
# fused path: clefq_tp_mlp over a TpComm (stores into peers' regions, device barriers)
# ---------------------------------------------------------------------------------------
def test_tp_region_and_workspace_sizes():
    """Host-side shape arithmetic of the fused path (no device work)."""
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    import clefq
    L = clefq.lib()
    m, h, i = 4096, 4096, 12288
    for world in (1, 2, 4, 8):
        region = L.clefq_tp_mlp_region_bytes(m, h, i, world)
        assert region >= world * m * 4 + m * i // 2 + m * h * 2   # maxima, int4 codes, output
        assert L.clefq_tp_mlp_workspace_size(m, h, i, world) >= m * (2 * i // world) * 2
    assert L.clefq_tp_mlp_region_bytes(m, h, 12288 + 256, 2) == -1   # a 256-group would straddle ranks
    assert L.clefq_tp_mlp_region_bytes(m, 4096 + 256, i, 2) == -1     # odd 128-row tile count per rank
    assert L.clefq_tp_mlp_region_bytes(m, h, i, 9) == -1              # more ranks than one node


@pytest.mark.gpu
@pytest.mark.parametrize("m,residual", [(1, False), (129, True), (4096, True)])
def test_tp_fused_one_rank_matches_mlp(cq, m, residual):
    from clefq.tp import TpComm, mlp_tp_fused, shard_mlp, tp_mlp_region_bytes
    hidden, inter = 1024, 3072
    gate, up, down = _weights(cq, hidden, inter, 33)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(m + 1)
    with TpComm(tp_mlp_region_bytes(m, hidden, inter, 1)) as comm:
        shard = shard_mlp(gate, up, down, 0, 1)
        for rep in range(3):   # the barrier epochs advance across calls
            x = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16)
            res = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16) if residual else None
            out = mlp_tp_fused(x, shard, comm, residual=res)
            ref = cq.mlp(x, gate, up, down, residual=res)
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {rep}"
        cq.status()


@pytest.mark.gpu
def test_comm_barrier_times_out_without_peer(cq):
    """A two-rank group where rank 1 never arrives: rank 0's barrier gives up after the
    timeout, the status reports it, and the device keeps working."""
    L = cq.lib()
    c0, c1 = ctypes.c_void_p(), ctypes.c_void_p()
    cq._call("clefq_comm_create", 0, 2, 4096, ctypes.byref(c0), None)
    cq._call("clefq_comm_create", 1, 2, 4096, ctypes.byref(c1), None)
    try:
        assert L.clefq_comm_ready(c0) == 0
        cq._call("clefq_comm_attach", c0, 1, c1)
        assert L.clefq_comm_ready(c0) == 1
        cq._call("clefq_comm_set_timeout_ms", c0, 200)
        cq._call("clefq_comm_barrier", c0, cq._stream())
        with pytest.raises(RuntimeError, match="gave up"):
            cq.status()
        cq.status()   # the status word was cleared by the read
        x = torch.ones(4, 4, device="cuda")
        assert float((x @ x).sum()) == 64.0
    finally:
        torch.cuda.synchronize()
        cq._call("clefq_comm_destroy", c0)
        cq._call("clefq_comm_destroy", c1)


def _nccl_fused_worker(rank, world, port):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    import clefq as cq
    from clefq.tp import TpComm, mlp_tp_fused, shard_mlp, tp_mlp_region_bytes
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        hidden, inter = 2048, 8192
        gate, up, down = _weights(cq, hidden, inter, 9)
        shard = shard_mlp(gate, up, down, rank, world)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(5)                       # the same inputs on every rank
        with TpComm(tp_mlp_region_bytes(1000, hidden, inter, world)) as comm:
            for m in (1000, 7, 512):
                x = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16)
                res = torch.randn(m, hidden, device="cuda", generator=gen).to(torch.bfloat16)
                out = mlp_tp_fused(x, shard, comm, residual=res if m != 7 else None)
                ref = cq.mlp(x, gate, up, down, residual=res if m != 7 else None)
                assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"rank {rank} m {m}"
            cq.status()
            dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_fused_ranks_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_nccl_fused_worker, args=(world, _free_port()), nprocs=world, join=True,
                       start_method="spawn")
