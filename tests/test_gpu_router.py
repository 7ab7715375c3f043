"""clefq_route_linear: the Omni router linear (BF16 projection by mlp.gate) fused with the
router (src/omni.rs:760-765).

Two properties, as the kernel's contract states:
  * the routes are exactly omni_route of the logits the kernel reports: ids and BF16
    probabilities equal the CPU oracle's router (and the GPU router kernel) on those logits,
    bit for bit;
  * the logits are the BF16 projection within one BF16 rounding step of an exact (float64)
    dot product -- the f32 accumulation order is the kernel's own, as any GEMM's is.
Inputs follow BASELINE configs[3]: hidden rows and router weight BF16 N(0, 1).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as o
from tests.gpu_util import bf16_normal, from_dev_bf16, same_bits_f32, to_dev_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cq():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import clefq
    clefq.lib()
    return clefq


def _check(cq, x, w, topk):
    routes, logits = cq.omni_route_linear(to_dev_bf16(x), to_dev_bf16(w), topk, logits_out=True)
    lg = from_dev_bf16(logits)
    rt = routes.cpu().numpy()
    # routes == the reference router on the reported logits (CPU oracle and the GPU router)
    assert same_bits_f32(rt, o.route(lg, topk))
    assert same_bits_f32(rt, cq.omni_route(logits, topk).cpu().numpy())
    # logits: within one BF16 step of the exact dot product
    exact = o.bf16_to_f32(x).astype(np.float64) @ o.bf16_to_f32(w).astype(np.float64).T
    got = o.bf16_to_f32(lg).astype(np.float64)
    tol = np.abs(exact) * 2.0 ** -7 + 1e-3
    assert np.all(np.abs(got - exact) <= tol), float(np.max(np.abs(got - exact) - tol))
    same = np.mean(lg == o.f32_to_bf16(exact.astype(np.float32)))
    assert same > 0.98, same
    return rt, lg


@pytest.mark.parametrize("tokens,hidden,experts,topk", [
    (1, 2048, 128, 8), (100, 2048, 128, 8), (1000, 512, 64, 4), (8192, 2048, 128, 8), (300, 1024, 96, 8),
    (129, 256, 32, 2)])
def test_route_linear_matches_router_on_its_logits(cq, tokens, hidden, experts, topk):
    rng = np.random.default_rng(tokens + hidden + experts)
    x = bf16_normal(rng, (tokens, hidden))
    w = bf16_normal(rng, (experts, hidden))
    for _ in range(2):
        _check(cq, x, w, topk)
    cq.status()


def test_route_linear_ties_and_degenerate_rows(cq):
    """Zero rows (all logits 0: ties ranked by ascending id), rows whose logits are all equal
    after BF16 rounding, and very large inputs."""
    rng = np.random.default_rng(7)
    tokens, hidden, experts = 64, 512, 128
    x = bf16_normal(rng, (tokens, hidden))
    x[0] = 0
    x[1] = o.f32_to_bf16(np.full(hidden, 1e-30, np.float32))
    x[2] = o.f32_to_bf16(np.full(hidden, 3e4, np.float32))
    w = bf16_normal(rng, (experts, hidden))
    w[5] = w[9]                      # two experts with identical weights: tied logits on every row
    rt, _ = _check(cq, x, w, 8)
    assert list(rt[0, :8]) == list(range(8))
    assert np.all(rt[0, 8:] == np.float32(0.125))


def test_route_linear_rejects_bad_shapes(cq):
    x = torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((128, 100), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        cq.omni_route_linear(x, w)
    x = torch.zeros((4, 256), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        cq.omni_route_linear(x, torch.zeros((100, 256), dtype=torch.bfloat16, device="cuda"))


def _expert_weights(cq, rng, experts, n, k):
    w = bf16_normal(rng, (experts * n, k), 0.05)
    wt, ws = o.pack_weight(w)
    from tests.gpu_util import to_dev
    return (wt, ws), cq.QuantizedWeight(to_dev(wt.view(np.int32)), to_dev(ws), experts * n, k, o.stride_for(k), 4)


def test_moe_block_with_fused_router(cq):
    """clefq_moe given the router weight (CLEFQ_ROUTER_WEIGHT_BF16) equals the oracle's MoE
    block on the logits the fused router reports, bit for bit; so does the one-rank fused
    expert-parallel layer."""
    from clefq.comm import Comm
    from clefq.ep import ep_layer_region_bytes, omni_moe_ep_fused, shard_experts
    rng = np.random.default_rng(21)
    tokens, experts, topk, hidden, inter = 300, 128, 8, 512, 256
    (gt, gs), gdev = _expert_weights(cq, rng, experts, inter, hidden)
    (ut, us), udev = _expert_weights(cq, rng, experts, inter, hidden)
    (dt, ds), ddev = _expert_weights(cq, rng, experts, hidden, inter)
    x = bf16_normal(rng, (tokens, hidden))
    wr = bf16_normal(rng, (experts, hidden))
    xd, wd = to_dev_bf16(x), to_dev_bf16(wr)
    _, logits = cq.omni_route_linear(xd, wd, topk, logits_out=True)
    ref, ref_routes, _, _ = o.moe_layer(x, from_dev_bf16(logits), (gt, gs, inter), (ut, us, inter), (dt, ds, hidden))
    routes = torch.empty((tokens, 2 * topk), dtype=torch.float32, device="cuda")
    for _ in range(2):
        out = cq.omni_moe(xd, None, gdev, udev, ddev, router_weight=wd, routes_out=routes)
        assert same_bits_f32(routes.cpu().numpy(), ref_routes)
        assert np.array_equal(from_dev_bf16(out), ref)
    shard = shard_experts(gdev, udev, ddev, experts, inter, hidden, 0, 1)
    with Comm(ep_layer_region_bytes(tokens, hidden, topk, 1, tokens * topk)) as comm:
        out, ep_routes = omni_moe_ep_fused(xd, None, shard, comm, topk, router_weight=wd)
        assert same_bits_f32(ep_routes.cpu().numpy(), ref_routes)
        assert np.array_equal(from_dev_bf16(out), ref)
    cq.status()
