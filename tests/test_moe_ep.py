"""Expert-parallel Omni MoE: every rank's output equals the single-GPU layer bit for bit.

- CPU, 2 and 4 gloo ranks: the real host orchestration (clefq.ep.omni_moe_ep) with the device
  steps replaced by oracle stand-ins, against the oracle's single-process moe_layer
  (src/omni.rs:761-857 semantics).
- GPU, one process: G = 2 and 4 ranks simulated by splicing send/receive buffers exactly as
  the two all-to-all exchanges do, through every libclefq expert-parallel entry point,
  against clefq.omni_moe on the same tokens.
- GPU, 2 processes over NCCL (needs two GPUs).
"""
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
# CPU: 2 gloo ranks, oracle stand-ins
# ---------------------------------------------------------------------------------------
CPU_T, CPU_H, CPU_I, CPU_E, CPU_K = 24, 256, 256, 8, 2


def _cpu_problem(world):
    from oracle import oracle as o
    rng = np.random.default_rng(7)
    x = o.f32_to_bf16(rng.standard_normal((world * CPU_T, CPU_H)).astype(np.float32))
    logits = o.f32_to_bf16(rng.standard_normal((world * CPU_T, CPU_E)).astype(np.float32))
    gate = o.pack_weight(o.f32_to_bf16(rng.standard_normal((CPU_E * CPU_I, CPU_H)).astype(np.float32) * 0.05))
    up = o.pack_weight(o.f32_to_bf16(rng.standard_normal((CPU_E * CPU_I, CPU_H)).astype(np.float32) * 0.05))
    down = o.pack_weight(o.f32_to_bf16(rng.standard_normal((CPU_E * CPU_H, CPU_I)).astype(np.float32) * 0.05))
    return x, logits, gate, up, down


def _cpu_worker(rank, world, port):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    from oracle import oracle as o
    from clefq.ep import ExpertShard, omni_moe_ep
    from tests.ep_oracle_ops import OracleEpOps
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x, logits, gate, up, down = _cpu_problem(world)
        per = CPU_E // world
        base = rank * per

        def cut(w, rows_per_expert, cols):
            words = cols // 8
            lo, hi = base * rows_per_expert, (base + per) * rows_per_expert
            return (w[0][lo * words:hi * words], w[1][lo:hi])
        shard = ExpertShard(cut(gate, CPU_I, CPU_H), cut(up, CPU_I, CPU_H), cut(down, CPU_H, CPU_I), base, per, CPU_E,
                            CPU_I)
        mine = slice(rank * CPU_T, (rank + 1) * CPU_T)
        xt = torch.from_numpy(x[mine].view(np.int16).copy()).view(torch.bfloat16)
        lt = torch.from_numpy(logits[mine].view(np.int16).copy()).view(torch.bfloat16)
        out, routes = omni_moe_ep(xt, lt, shard, CPU_K, ops=OracleEpOps())
        # weight tuples: (tiled codes, scales, rows per expert)
        ref, ref_routes, _, _ = o.moe_layer(x, logits, (gate[0], gate[1], CPU_I), (up[0], up[1], CPU_I),
                                            (down[0], down[1], CPU_H), CPU_K, CPU_E)
        got = out.view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(routes.numpy(), ref_routes[mine])
        assert np.array_equal(got, ref[mine]), f"rank {rank}: {np.count_nonzero(got != ref[mine])} mismatches"
    finally:
        dist.destroy_process_group()


def test_ep_host_logic_two_gloo_ranks():
    mp.start_processes(_cpu_worker, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")


def _abandon_worker(rank, world, port):
    """Rank 1 leaves between layers (after joining the group, before the layer's first
    exchange); rank 0's layer must end with an error from the process group -- its peer's
    closed connection or the group's 5 s timeout -- instead of waiting for good."""
    import datetime
    import time
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    from clefq.ep import ExpertShard, omni_moe_ep
    from tests.ep_oracle_ops import OracleEpOps
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        return
    x, logits, gate, up, down = _cpu_problem(world)
    per = CPU_E // world

    def cut(w, rows_per_expert, cols):
        words = cols // 8
        return (w[0][: per * rows_per_expert * words], w[1][: per * rows_per_expert])
    shard = ExpertShard(cut(gate, CPU_I, CPU_H), cut(up, CPU_I, CPU_H), cut(down, CPU_H, CPU_I), 0, per, CPU_E, CPU_I)
    xt = torch.from_numpy(x[:CPU_T].view(np.int16).copy()).view(torch.bfloat16)
    lt = torch.from_numpy(logits[:CPU_T].view(np.int16).copy()).view(torch.bfloat16)
    t0 = time.monotonic()
    try:
        omni_moe_ep(xt, lt, shard, CPU_K, ops=OracleEpOps())
    except RuntimeError:
        assert time.monotonic() - t0 < 60
    else:
        raise AssertionError("the expert-parallel layer finished without its peer")


def test_ep_departed_rank_ends_layer_with_error():
    mp.start_processes(_abandon_worker, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")


def test_ep_host_logic_four_gloo_ranks():
    """Four ranks, two experts each: uneven counts per rank pair, every rank bit-exact."""
    mp.start_processes(_cpu_worker, args=(4, _free_port()), nprocs=4, join=True, start_method="spawn")


def test_ep_record_bytes_matches_library_formula():
    from tests.ep_oracle_ops import record_bytes
    import clefq
    for h in (256, 2048, 4096, 7168):
        assert clefq.lib().clefq_moe_ep_record_bytes(h) == record_bytes(h)


# ---------------------------------------------------------------------------------------
# GPU, one process: simulated ranks
# ---------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cq():
    import clefq
    clefq.lib()
    return clefq


def _weights(cq, experts, inter, hidden, seed):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)

    def w(rows, cols):
        return cq.load_quantized_weight((torch.randn(rows, cols, device="cuda", generator=gen) * 0.05)
                                        .to(torch.bfloat16))
    return w(experts * inter, hidden), w(experts * inter, hidden), w(experts * hidden, inter)


@pytest.mark.gpu
@pytest.mark.parametrize("world,experts,topk,tokens,hidden,inter", [
    (2, 16, 4, 100, 512, 256), (4, 16, 4, 37, 512, 256), (4, 128, 8, 300, 512, 256),
    (2, 128, 8, 1000, 2048, 768), (4, 64, 8, 333, 2048, 768), (2, 128, 8, 8192, 2048, 768)])
def test_ep_simulated_ranks_match_single_gpu(cq, world, experts, topk, tokens, hidden, inter):
    """Hidden 2048 takes the deep-ring kernel for the expert gate|up GEMM (K >= 2048), 512
    the two-stage kernel."""
    from clefq.ep import CudaEpOps, shard_experts
    gate, up, down = _weights(cq, experts, inter, hidden, 11)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(world * 100 + tokens)
    xs = [torch.randn(tokens + 3 * h, hidden, device="cuda", generator=gen).to(torch.bfloat16) for h in range(world)]
    ls = [torch.randn(tokens + 3 * h, experts, device="cuda", generator=gen).to(torch.bfloat16) for h in range(world)]
    shards = [shard_experts(gate, up, down, experts, inter, hidden, d, world) for d in range(world)]
    ops = CudaEpOps()
    rec = ops.record_bytes(hidden)
    home = []
    for h in range(world):
        routes = ops.route(ls[h], topk)
        codes, scales = ops.pack_tokens(xs[h])
        counts, slots = ops.plan(routes, topk, experts, world)
        sc = counts.tolist()
        send = ops.pack_records(codes, scales, routes, topk, slots, sum(sc), hidden)
        home.append((routes, slots, sc, send))
    # first all-to-all: destination d receives, from every source in rank order, its slice
    products = []
    for d in range(world):
        parts, rc = [], []
        for h in range(world):
            sc = home[h][2]
            lo = sum(sc[:d]) * rec
            parts.append(home[h][3][lo:lo + sc[d] * rec])
            rc.append(sc[d])
        recv = torch.cat(parts) if sum(rc) else torch.empty(rec, dtype=torch.uint8, device="cuda")
        products.append((ops.experts(recv, sum(rc), hidden, shards[d]), rc))
    # second all-to-all: home h gets, from every destination in rank order, its products
    for h in range(world):
        routes, slots, sc, _ = home[h]
        back = torch.cat([products[d][0][sum(products[d][1][:h]):sum(products[d][1][:h]) + sc[d]]
                          for d in range(world)])
        out = ops.combine(back, slots, routes, topk, hidden)
        ref_routes = torch.empty(xs[h].shape[0], 2 * topk, dtype=torch.float32, device="cuda")
        ref = cq.omni_moe(xs[h], ls[h], gate, up, down, experts=experts, topk=topk, routes_out=ref_routes)
        assert torch.equal(routes, ref_routes)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (
            f"home {h}: {(out.view(torch.int16) != ref.view(torch.int16)).sum().item()} mismatches")


# ---------------------------------------------------------------------------------------
# GPU, 2 processes over NCCL
# ---------------------------------------------------------------------------------------
def _nccl_worker(rank, world, port, hidden=512, inter=256):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    import clefq as cq
    from clefq.ep import omni_moe_ep, shard_experts
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        experts, topk, tokens = 32, 8, 257 + 31 * rank
        gate, up, down = _weights(cq, experts, inter, hidden, 5)
        shard = shard_experts(gate, up, down, experts, inter, hidden, rank, world)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(1000 + rank)
        x = torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16)
        logits = torch.randn(tokens, experts, device="cuda", generator=gen).to(torch.bfloat16)
        out, routes = omni_moe_ep(x, logits, shard, topk)
        ref = cq.omni_moe(x, logits, gate, up, down, experts=experts, topk=topk)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("hidden,inter", [(512, 256), (2048, 768)])
def test_ep_ranks_nccl(world, hidden, inter):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_nccl_worker, args=(world, _free_port(), hidden, inter), nprocs=world, join=True,
                       start_method="spawn")


# ---------------------------------------------------------------------------------------
# fused path: clefq_moe_ep_layer over a Comm (records and products stored into peers)
# ---------------------------------------------------------------------------------------
@pytest.mark.gpu
@pytest.mark.parametrize("experts,topk,tokens,hidden,inter", [
    (16, 4, 100, 512, 256), (128, 8, 300, 512, 256), (32, 8, 1, 512, 256), (128, 8, 1000, 2048, 768)])
def test_ep_fused_one_rank_matches_moe(cq, experts, topk, tokens, hidden, inter):
    from clefq.comm import Comm
    from clefq.ep import ep_layer_region_bytes, omni_moe_ep_fused, shard_experts
    gate, up, down = _weights(cq, experts, inter, hidden, 17)
    shard = shard_experts(gate, up, down, experts, inter, hidden, 0, 1)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(tokens)
    with Comm(ep_layer_region_bytes(tokens, hidden, topk, 1, tokens * topk)) as comm:
        for rep in range(3):   # barrier epochs and buffers reused across calls
            x = torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16)
            logits = torch.randn(tokens, experts, device="cuda", generator=gen).to(torch.bfloat16)
            out, routes = omni_moe_ep_fused(x, logits, shard, comm, topk)
            ref_routes = torch.empty(tokens, 2 * topk, dtype=torch.float32, device="cuda")
            ref = cq.omni_moe(x, logits, gate, up, down, experts=experts, topk=topk, routes_out=ref_routes)
            assert torch.equal(routes, ref_routes)
            assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"call {rep}"
        cq.status()


@pytest.mark.gpu
def test_ep_fused_one_rank_full_size(cq):
    """The fused layer at BASELINE configs[3] size on one rank (8192 tokens, hidden 2048, inter 768,
    128 experts, top-8), with the benchmark's inputs: random int4 weight words, logits of
    BF16 N(0, 1) rows through a BF16 N(0, 1) router weight.  Repeated calls and a receive
    capacity above the routes present; every call bit-identical to clefq_moe."""
    from clefq.comm import Comm
    from clefq.ep import ep_layer_region_bytes, omni_moe_ep_fused, shard_experts
    tokens, hidden, inter, experts, topk = 8192, 2048, 768, 128, 8
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2000)

    def rand_weight(rows, cols):
        codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows * cols // 8,), dtype=torch.int32, device="cuda",
                              generator=gen)
        scales = (torch.randn(rows, device="cuda", generator=gen).abs() * 0.02 / 7).float()
        return cq.QuantizedWeight(codes, scales, rows, cols, cq.stride_for(cols), 4)
    gate, up = rand_weight(experts * inter, hidden), rand_weight(experts * inter, hidden)
    down = rand_weight(experts * hidden, inter)
    x = torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16)
    wr = torch.randn(experts, hidden, device="cuda", generator=gen).to(torch.bfloat16)
    logits = x @ wr.t()
    ref = cq.omni_moe(x, logits, gate, up, down)
    shard = shard_experts(gate, up, down, experts, inter, hidden, 0, 1)
    for cap in (tokens * topk, 2 * tokens * topk):
        with Comm(ep_layer_region_bytes(tokens, hidden, topk, 1, cap)) as comm:
            for rep in range(3):
                out, _ = omni_moe_ep_fused(x, logits, shard, comm, topk, recv_cap=cap)
                bad = int((out.view(torch.int16) != ref.view(torch.int16)).sum())
                assert bad == 0, f"capacity {cap}, call {rep}: {bad} outputs differ"
    cq.status()


@pytest.mark.gpu
def test_ep_fused_capacity_overflow_is_reported(cq):
    """A receive capacity below the routes present: the excess records are dropped, the
    status reports it on the host, and the device keeps working."""
    from clefq.comm import Comm
    from clefq.ep import ep_layer_region_bytes, omni_moe_ep_fused, shard_experts
    experts, topk, hidden, inter, tokens = 16, 4, 512, 256, 64
    gate, up, down = _weights(cq, experts, inter, hidden, 3)
    shard = shard_experts(gate, up, down, experts, inter, hidden, 0, 1)
    x = torch.randn(tokens, hidden, device="cuda").to(torch.bfloat16)
    logits = torch.randn(tokens, experts, device="cuda").to(torch.bfloat16)
    cap = tokens * topk // 2
    with Comm(ep_layer_region_bytes(tokens, hidden, topk, 1, cap)) as comm:
        omni_moe_ep_fused(x, logits, shard, comm, topk, recv_cap=cap)
        with pytest.raises(RuntimeError, match="gave up"):
            cq.status()
        out, _ = omni_moe_ep_fused(x, logits, shard, comm, topk, recv_cap=cap)
        with pytest.raises(RuntimeError):
            cq.status()
    ref = cq.omni_moe(x, logits, gate, up, down, experts=experts, topk=topk)
    assert ref.shape == out.shape
    cq.status()


def _nccl_fused_worker(rank, world, port, hidden=512, inter=256):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "clef-hrx_b200"))
    import clefq as cq
    from clefq.comm import Comm
    from clefq.ep import ep_layer_region_bytes, omni_moe_ep_fused, shard_experts
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        experts, topk = 32, 8
        most = 257 + 31 * (world - 1)
        cap = world * most * topk                   # the same on every rank
        gate, up, down = _weights(cq, experts, inter, hidden, 5)
        shard = shard_experts(gate, up, down, experts, inter, hidden, rank, world)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(1000 + rank)
        with Comm(ep_layer_region_bytes(most, hidden, topk, world, cap)) as comm:
            for rep in range(3):
                tokens = 257 + 31 * rank - 100 * rep   # ranks and calls differ in token count
                x = torch.randn(tokens, hidden, device="cuda", generator=gen).to(torch.bfloat16)
                logits = torch.randn(tokens, experts, device="cuda", generator=gen).to(torch.bfloat16)
                out, routes = omni_moe_ep_fused(x, logits, shard, comm, topk, recv_cap=cap)
                ref = cq.omni_moe(x, logits, gate, up, down, experts=experts, topk=topk)
                assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"rank {rank} call {rep}"
            cq.status()
            dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("hidden,inter", [(512, 256), (2048, 768)])
def test_ep_fused_ranks(world, hidden, inter):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_nccl_fused_worker, args=(world, _free_port(), hidden, inter), nprocs=world, join=True,
                       start_method="spawn")
