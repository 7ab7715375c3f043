"""GPU parity at the benchmarked sizes: BASELINE configs C1-C4 at their full shapes through the
C ABI, against the CPU oracle, bit for bit.

Inputs follow the BASELINE distributions (seeded): activations BF16 N(0, 1); weight codes
uniform in [-8, 7] (uniform random tiled words, so -8 occurs, which the reference's packer
never emits but its GEMM fixture does); one f32 scale per output row |N(0, 0.02)|/7; router
logits from a BF16 N(0, 1) router weight.  These are the shapes bench.py times, so the
deep-ring dense kernel at K=4096/12288 with its per-tile K rotation, partial last wave and
SwiGLU epilogue, and the grouped expert kernels at the C4 per-expert tile counts, are all
checked here.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as o
from tests.gpu_util import bf16_normal, from_dev_bf16, same_bits_f32, to_dev, to_dev_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cq():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import clefq
    clefq.lib()
    return clefq


def baseline_weight(cq, rng, rows, cols):
    """BASELINE weight: random tiled int4 words (codes uniform in [-8, 7]), scales |N(0,0.02)|/7.
    Returns the oracle tuple (tiled words, scales, rows) and the device QuantizedWeight."""
    words = rng.integers(0, 2 ** 32, size=rows * cols // 8, dtype=np.uint64).astype(np.uint32)
    scales = (np.abs(rng.standard_normal(rows)) * 0.02 / 7).astype(np.float32)
    dev = cq.QuantizedWeight(to_dev(words.view(np.int32)), to_dev(scales), rows, cols, o.stride_for(cols), 4)
    return (words, scales, rows), dev


def test_c1_single_gemm(cq):
    """C1: 128 x 2048 activations through a 768 x 2048 weight, BF16 and F32 outputs."""
    rng = np.random.default_rng(0)
    m, k, n = 128, 2048, 768
    w, wdev = baseline_weight(cq, rng, n, k)
    x = bf16_normal(rng, (m, k))
    _, codes, scales, _ = o.prepare(x, 4, o.stride_for(k))
    a = cq.prepare(to_dev_bf16(x), 4, o.stride_for(k))
    for _ in range(2):
        assert np.array_equal(from_dev_bf16(cq.project_prepared(m, wdev, a)), o.gemm(codes, scales, w[0], w[1], n, k))
        out32 = cq.project_prepared(m, wdev, a, out_dtype=torch.float32)
        assert same_bits_f32(out32.cpu().numpy(), o.gemm(codes, scales, w[0], w[1], n, k, out_f32=True))


def test_c2_mlp_block_full_size(cq):
    """C2: the whole dense SwiGLU MLP block, 4096 tokens, 4096 -> 12288 -> 4096, one clefq_mlp
    call against the oracle's separate steps."""
    rng = np.random.default_rng(2)
    m, h, inter = 4096, 4096, 12288
    g, gdev = baseline_weight(cq, rng, inter, h)
    u, udev = baseline_weight(cq, rng, inter, h)
    d, ddev = baseline_weight(cq, rng, h, inter)
    x = bf16_normal(rng, (m, h))
    ref = o.mlp_block(x, g, u, d)
    xd = to_dev_bf16(x)
    ws = torch.empty(cq.lib().clefq_mlp_workspace_size(m, h, inter), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        out = cq.mlp(xd, gdev, udev, ddev, workspace=ws)
        got = from_dev_bf16(out)
        assert np.array_equal(got, ref), f"{int((got != ref).sum())} of {ref.size} outputs differ"
    cq.status()


def test_c2_gate_up_pair_and_down_full_size(cq):
    """C2's GEMM launches: gate|up as one paired launch (N = 2 x 12288, two weight maps), plain
    and with SwiGLU in the epilogue as clefq_mlp issues it, and the down projection (K = 12288)
    with F32 output and with a BF16 residual."""
    rng = np.random.default_rng(3)
    m, h, inter = 4096, 4096, 12288
    g, gdev = baseline_weight(cq, rng, inter, h)
    u, udev = baseline_weight(cq, rng, inter, h)
    x = bf16_normal(rng, (m, h))
    _, codes, scales, _ = o.prepare(x, 4, o.stride_for(h))
    a = cq.prepare(to_dev_bf16(x), 4, o.stride_for(h))
    pair = from_dev_bf16(cq.project_pair_prepared(m, gdev, udev, a))
    gate_ref = o.gemm(codes, scales, g[0], g[1], inter, h)
    up_ref = o.gemm(codes, scales, u[0], u[1], inter, h)
    assert np.array_equal(pair[:, :inter], gate_ref)
    assert np.array_equal(pair[:, inter:], up_ref)
    # the same launch with SwiGLU in its epilogue, as clefq_mlp issues it at this shape
    fused = from_dev_bf16(cq.project_swiglu_prepared(m, gdev, udev, a))
    assert np.array_equal(fused, o.swiglu(gate_ref, up_ref))

    d, ddev = baseline_weight(cq, rng, h, inter)
    hid = bf16_normal(rng, (m, inter))
    res = bf16_normal(rng, (m, h))
    _, hc, hs, _ = o.prepare(hid, 4, o.stride_for(inter))
    b = cq.prepare(to_dev_bf16(hid), 4, o.stride_for(inter))
    out32 = cq.project_prepared(m, ddev, b, out_dtype=torch.float32)
    assert same_bits_f32(out32.cpu().numpy(), o.gemm(hc, hs, d[0], d[1], h, inter, out_f32=True))
    outr = cq.project_prepared(m, ddev, b, residual=to_dev_bf16(res))
    assert np.array_equal(from_dev_bf16(outr), o.gemm(hc, hs, d[0], d[1], h, inter, residual=res))
    cq.status()


@pytest.mark.parametrize("n,k", [(4096, 2560), (1024, 2560), (2560, 4096)])
def test_c3_attention_projections(cq, n, k):
    """C3's q, k/v and o projections at S = 2048 (hidden 2560: no stride padding, 10 pair
    tiles across for o)."""
    rng = np.random.default_rng(n + k)
    m = 2048
    w, wdev = baseline_weight(cq, rng, n, k)
    x = bf16_normal(rng, (m, k))
    _, codes, scales, _ = o.prepare(x, 4, o.stride_for(k))
    out = cq.project_quantized(to_dev_bf16(x), wdev)
    assert np.array_equal(from_dev_bf16(out), o.gemm(codes, scales, w[0], w[1], n, k))


def test_c3_normalized_mlp(cq):
    """C3's MLP: RMSNorm (weights 1 + N(0, 0.02)) fused into the packing, 2560 -> 9728 -> 2560,
    the un-normalised input as residual (normalized_mlp, src/quantized.rs:348-404)."""
    rng = np.random.default_rng(7)
    m, h, inter = 2048, 2560, 9728
    g, gdev = baseline_weight(cq, rng, inter, h)
    u, udev = baseline_weight(cq, rng, inter, h)
    d, ddev = baseline_weight(cq, rng, h, inter)
    x = bf16_normal(rng, (m, h))
    # the stored norm weight is w with the reference's +1 offset applied in the kernel
    nw = o.f32_to_bf16((rng.standard_normal(h) * 0.02).astype(np.float32))
    ref = o.normalized_mlp_block(x, nw, g, u, d)
    xd = to_dev_bf16(x)
    for _ in range(2):
        out = cq.normalized_mlp(xd, to_dev_bf16(nw), gdev, udev, ddev)
        assert np.array_equal(from_dev_bf16(out), ref)
    inplace = xd.clone()
    cq.normalized_mlp(inplace, to_dev_bf16(nw), gdev, udev, ddev, out=inplace)
    assert np.array_equal(from_dev_bf16(inplace), ref)
    cq.status()


def test_c4_moe_layer_full_size(cq):
    """C4: the Omni MoE layer at 8192 tokens, hidden 2048, 128 experts x (gate|up 2048 -> 2 x 768,
    down 768 -> 2048), top-8, logits from a BF16 N(0, 1) router weight: routes, and the
    combined output, bit for bit."""
    rng = np.random.default_rng(4)
    t, h, inter, e = 8192, 2048, 768, 128
    g, gdev = baseline_weight(cq, rng, e * inter, h)
    u, udev = baseline_weight(cq, rng, e * inter, h)
    d, ddev = baseline_weight(cq, rng, e * h, inter)
    x = bf16_normal(rng, (t, h))
    wr = bf16_normal(rng, (e, h))
    logits = o.f32_to_bf16(o.bf16_to_f32(x) @ o.bf16_to_f32(wr).T)
    ref, ref_routes, ref_groups, _ = o.moe_layer(x, logits, (g[0], g[1], inter), (u[0], u[1], inter),
                                                 (d[0], d[1], h))
    counts = ref_groups[:, 0]
    assert counts.sum() == t * 8 and counts.max() > counts.min()   # uneven expert loads
    routes_out = torch.empty((t, 16), dtype=torch.float32, device="cuda")
    xd, ld = to_dev_bf16(x), to_dev_bf16(logits)
    ws = torch.empty(cq.lib().clefq_moe_workspace_size(t, h, inter, e, 8), dtype=torch.uint8, device="cuda")
    for _ in range(2):
        out = cq.omni_moe(xd, ld, gdev, udev, ddev, workspace=ws, routes_out=routes_out)
        assert same_bits_f32(routes_out.cpu().numpy(), ref_routes)
        got = from_dev_bf16(out)
        assert np.array_equal(got, ref), f"{int((got != ref).sum())} of {ref.size} outputs differ"
    cq.status()


@pytest.mark.parametrize("tokens,inter,skewed", [(8192, 768, False), (300, 256, True), (1, 512, False)])
def test_fused_gate_up_experts(cq, tokens, inter, skewed):
    """omni_gate_up (src/omni.rs:302-373): gate and up experts with SwiGLU in the GEMM epilogue,
    against the oracle's two expert projections and SwiGLU, bit for bit (C4 shape first)."""
    from tests.golden.make_golden import expert_routes
    rng = np.random.default_rng(tokens + inter)
    hidden, experts = 2048, 128
    g, gdev = baseline_weight(cq, rng, experts * inter, hidden)
    u, udev = baseline_weight(cq, rng, experts * inter, hidden)
    if tokens == 8192:
        x = bf16_normal(rng, (tokens, hidden))
        wr = bf16_normal(rng, (experts, hidden))
        routes = o.route(o.f32_to_bf16(o.bf16_to_f32(x) @ o.bf16_to_f32(wr).T))
    else:
        x = bf16_normal(rng, (tokens, hidden))
        routes = expert_routes(tokens, skewed, 0)
    groups, _ = o.group(routes)
    _, xc, xs, _ = o.prepare(x, 4, o.stride_for(hidden))
    gate_ref = o.expert(xc, xs, g[0], g[1], groups, tokens, hidden, inter, False)
    up_ref = o.expert(xc, xs, u[0], u[1], groups, tokens, hidden, inter, False)
    ref = o.swiglu(gate_ref, up_ref)
    a = cq.prepare(to_dev_bf16(x), 4, o.stride_for(hidden))
    for _ in range(2):
        out = cq.omni_gate_up(a, to_dev(routes), to_dev(groups), gdev, udev)
        got = from_dev_bf16(out)
        assert np.array_equal(got, ref), f"{int((got != ref).sum())} of {ref.size} differ"
    cq.status()
