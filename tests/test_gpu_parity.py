"""GPU parity: the sm_100a kernels through the C ABI against the CPU oracle, bit for bit.

Integer accumulators, codes, scales, routing ids, groupings and combine outputs are
bit-exact; the BF16 epilogues are bit-exact too because both sides round identically and
share one exp algorithm.  Every case runs twice on the device (replay determinism, as in
the reference tests).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as o
from tests.gpu_util import (bf16_equal_nan, bf16_normal, from_dev_bf16, permuted_operand, same_bits_f32, to_dev,
                            to_dev_bf16)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cq():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import clefq
    clefq.lib()
    return clefq


def _dev_prepared(cq, x_np, bits, stride, kind=0, aux=None):
    x = to_dev_bf16(x_np)
    a = None if aux is None else to_dev_bf16(aux)
    return cq.prepare(x, bits, stride, kind, a)


def _words(p):
    return p.codes.cpu().numpy().view(np.uint32)


# ---------------------------------------------------------------------------------------
# packing
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("width", [256, 768, 1280, 5120, 6144, 8192, 17408])
def test_prepare_matches_golden(cq, golden, bits, width):
    key = f"pack_b{bits}_w{width}"
    x = golden[key + "_x"]
    stride = width + 512 // bits
    for _ in range(2):
        p = _dev_prepared(cq, x, bits, stride)
        words = _words(p)
        assert np.array_equal(words[:, : width // (32 // bits)], golden[key + "_words"])
        assert not np.any(words[:, width // (32 // bits):]), "stride padding must be zero"
        _, _, oscales, _ = o.prepare(x, bits, stride)
        assert same_bits_f32(p.scales.cpu().numpy(), oscales)
        if bits == 4:
            assert np.array_equal(p.operand.cpu().numpy(), permuted_operand(words, width))


@pytest.mark.parametrize("bits", [4, 8])
def test_prepare_exceptional_rows(cq, golden, bits):
    x = golden[f"exc_b{bits}_x"]
    p = _dev_prepared(cq, x, bits, 5120 + 512 // bits)
    assert np.array_equal(_words(p)[:, : 5120 // (32 // bits)], golden[f"exc_b{bits}_words"])
    assert same_bits_f32(p.scales.cpu().numpy(), golden[f"exc_b{bits}_scales"])


@pytest.mark.parametrize("rows,width", [(1, 256), (7, 768), (33, 2048), (130, 4096), (5, 12288), (3, 32768)])
@pytest.mark.parametrize("bits", [4, 8])
def test_prepare_random_matches_oracle(cq, rows, width, bits):
    rng = np.random.default_rng(rows * 7 + width)
    x = bf16_normal(rng, (rows, width))
    stride = o.stride_for(width, bits)
    p = _dev_prepared(cq, x, bits, stride)
    storage, _, _, _ = o.prepare(x, bits, stride)
    assert np.array_equal(p.storage.cpu().numpy().view(np.uint32), storage)


@pytest.mark.parametrize("rows,width", [(1, 256), (7, 768), (300, 2048), (130, 4096), (65, 12288), (3, 32768)])
def test_prepare_codes_only_matches_oracle(cq, rows, width):
    """Plain int4 packing without the s8 operand (weights, expert-parallel tokens) takes the
    persistent packing kernel where it fits; codes, stride padding and scales stay exact."""
    rng = np.random.default_rng(rows * 3 + width)
    x = bf16_normal(rng, (rows, width), 1.7)
    x[0, 5] = 0x7FC0
    stride = o.stride_for(width)
    p = cq.prepare(to_dev_bf16(x), 4, stride, operand=False)
    storage, _, _, _ = o.prepare(x, 4, stride)
    assert np.array_equal(p.storage.cpu().numpy().view(np.uint32), storage)


def _gate_like(rng, rows, width):
    """SwiGLU/attention gate inputs with the reference test's exceptional rows
    (src/quantized.rs:1187-1266): 0, NaN, Inf, bf16 MAX, subnormal, +-80, formula."""
    i = np.arange(rows * width)
    col = i % width
    kind = (i // width) % 7
    v = ((i * 17 % 1031).astype(np.float32) - 515) / 16
    v = np.where(kind == 0, 0.0, v)
    v = np.where((kind == 1) & (col == 259), np.nan, v)
    v = np.where((kind == 2) & (col == 515), np.inf, v)
    v = np.where(kind == 3, o.bf16_to_f32(np.uint16(0x7F7F)), v)
    v = np.where(kind == 4, np.uint32(0x00010000).view(np.float32), v)
    v = np.where(kind == 5, np.where(col % 2 == 0, -80.0, 80.0), v)
    return o.f32_to_bf16(v.astype(np.float32)).reshape(rows, width)


@pytest.mark.parametrize("rows,width", [(9, 768), (14, 17408), (130, 2048)])
@pytest.mark.parametrize("bits", [4, 8])
def test_fused_swiglu_packing(cq, rows, width, bits):
    """Fused SwiGLU packing == oracle, and == the separate swiglu op + prepare
    (src/quantized.rs:1187-1266)."""
    rng = np.random.default_rng(width)
    g = _gate_like(rng, rows, width)
    i = np.arange(rows * width)
    u = o.f32_to_bf16(((i * 29 % 997).astype(np.float32) - 498) / 32).reshape(rows, width)
    stride = width + 512 // bits
    fused = _dev_prepared(cq, g, bits, stride, cq.PREP_SWIGLU, u)
    storage, _, _, _ = o.prepare(g, bits, stride, o.SWIGLU, u)
    assert np.array_equal(fused.storage.cpu().numpy().view(np.uint32), storage)
    act = cq.swiglu(to_dev_bf16(g), to_dev_bf16(u))
    assert bf16_equal_nan(from_dev_bf16(act), o.swiglu(g, u))
    sep = cq.prepare(act, bits, stride)
    assert torch.equal(sep.storage, fused.storage)


@pytest.mark.parametrize("rows,width", [(701, 768), (257, 1280), (300, 4096), (1201, 12288),
                                        (150, 20480), (70, 32768)])
@pytest.mark.parametrize("bits", [4, 8])
def test_swiglu_table_packing(cq, rows, width, bits):
    """Launches with at least a wave of groups take the SiLU-table kernel; every row count,
    group split and persistent-loop length must still equal the oracle bit for bit."""
    rng = np.random.default_rng(rows * 7 + width)
    g = _gate_like(rng, rows, width)
    u = bf16_normal(rng, (rows, width), 2.0)
    stride = width + 512 // bits
    fused = _dev_prepared(cq, g, bits, stride, cq.PREP_SWIGLU, u)
    storage, _, _, _ = o.prepare(g, bits, stride, o.SWIGLU, u)
    assert np.array_equal(fused.storage.cpu().numpy().view(np.uint32), storage)


@pytest.mark.parametrize("rows,width", [(3000, 4096), (4001, 512), (999, 1792)])
def test_plain_packing_many_row_blocks(cq, rows, width):
    """Plain packing over more row blocks than resident CTAs (prefetch across iterations)."""
    rng = np.random.default_rng(rows)
    x = bf16_normal(rng, (rows, width), 1.5)
    stride = o.stride_for(width)
    p = _dev_prepared(cq, x, 4, stride, cq.PREP_PLAIN, None)
    storage, _, _, _ = o.prepare(x, 4, stride, o.PLAIN, None)
    assert np.array_equal(p.storage.cpu().numpy().view(np.uint32), storage)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("rows", [1, 158])
def test_attention_gate_packing(cq, bits, rows):
    """src/quantized.rs:1268-1368: Q halves are poisoned with NaN and must be ignored."""
    width = 6144
    rng = np.random.default_rng(rows)
    att = bf16_normal(rng, (rows, width), 4.0)
    q = _gate_like(rng, rows, 2 * width).copy()
    colq = np.arange(2 * width)
    q[:, (colq % 512) < 256] = 0x7FC0
    stride = width + 512 // bits
    p = _dev_prepared(cq, att, bits, stride, cq.PREP_ATTN_GATE, q)
    storage, _, _, _ = o.prepare(att, bits, stride, o.ATTN_GATE, q)
    assert np.array_equal(p.storage.cpu().numpy().view(np.uint32), storage)


@pytest.mark.parametrize("width", [5120, 2560])
def test_norm_packing(cq, width):
    rng = np.random.default_rng(width)
    rows = 37
    x = bf16_normal(rng, (rows, width), 3.0)
    w = bf16_normal(rng, (width,), 0.02)
    stride = o.stride_for(width)
    for kind, okind in ((cq.PREP_NORM, o.NORM), (cq.PREP_NORM_STORE, o.NORM_STORE)):
        p = _dev_prepared(cq, x, 4, stride, kind, w)
        storage, _, _, norm = o.prepare(x, 4, stride, okind, w)
        assert np.array_equal(p.storage.cpu().numpy().view(np.uint32), storage)
        if norm is not None:
            assert np.array_equal(from_dev_bf16(p.norm), norm)


@pytest.mark.parametrize("bits,rows,cols,padded", [(4, 256, 1024, True), (4, 384, 512, False),
                                                  (8, 128, 256, False), (4, 768, 2048, True)])
def test_retile(cq, bits, rows, cols, padded):
    stride = cols + (512 // bits if padded else 0)
    in_words = stride // (32 // bits)
    vals = (np.arange(rows * in_words, dtype=np.uint64) * 2654435761 % (1 << 32)).astype(np.uint32)
    vals = vals.reshape(rows, in_words)
    out = cq.retile_codes(to_dev(vals.view(np.int32)), rows, cols, bits)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), o.retile(vals, rows, cols, bits))


# ---------------------------------------------------------------------------------------
# dense GEMM
# ---------------------------------------------------------------------------------------
def _weight(rng, n, k, bits=4):
    w = bf16_normal(rng, (n, k), 0.05)
    wt, ws = o.pack_weight(w, bits)
    dev = cq_weight(wt, ws, n, k, bits)
    return w, wt, ws, dev


def cq_weight(wt, ws, n, k, bits):
    import clefq
    return clefq.QuantizedWeight(to_dev(wt.view(np.int32)), to_dev(ws), n, k, o.stride_for(k, bits), bits)


@pytest.mark.parametrize("m,n,k", [(1, 128, 256), (17, 256, 512), (127, 128, 2048), (128, 768, 2048),
                                   (129, 384, 1024), (300, 256, 4096), (64, 128, 12288)])
@pytest.mark.parametrize("bits", [4, 8])
def test_gemm_matches_oracle(cq, m, n, k, bits):
    rng = np.random.default_rng(m * 131 + n + k)
    _, wt, ws, wdev = _weight(rng, n, k, bits)
    x = bf16_normal(rng, (m, k))
    stride = o.stride_for(k, bits)
    _, ocodes, oscales, _ = o.prepare(x, bits, stride)
    ref, acc = o.gemm(ocodes, oscales, wt, ws, n, k, bits=bits, want_acc=True)
    ref32 = o.gemm(ocodes, oscales, wt, ws, n, k, bits=bits, out_f32=True)
    a = cq.prepare(to_dev_bf16(x), bits, stride)
    for _ in range(2):
        out = cq.project_prepared(m, wdev, a)          # s8 operand path (bits 4) / in-place (bits 8)
        assert np.array_equal(from_dev_bf16(out), ref)
    a_packed = cq.Prepared(a.storage, a.codes, a.scales, None, None, bits, stride)
    out2 = cq.project_prepared(m, wdev, a_packed)        # packed-codes path (unpack into workspace)
    assert np.array_equal(from_dev_bf16(out2), ref)
    out32 = cq.project_prepared(m, wdev, a, out_dtype=torch.float32)
    assert same_bits_f32(out32.cpu().numpy(), ref32)


@pytest.mark.parametrize("m", [1, 127, 256])
def test_gemm_residual(cq, m):
    """h3_gemm_i4_256_residual: bf16(res + bf16(y)), incl. NaN/Inf residuals and 1e34 scales
    (src/quantized.rs:1409-1552)."""
    rng = np.random.default_rng(m)
    n, k = 256, 1024
    _, wt, ws, wdev = _weight(rng, n, k)
    x = bf16_normal(rng, (m, k))
    res = bf16_normal(rng, (m, n))
    res[0, 0] = 0x7FC0
    res[0, 1] = 0x7F80
    x[0, :] = o.f32_to_bf16(np.full(k, 1e34, np.float32))
    stride = o.stride_for(k)
    _, ocodes, oscales, _ = o.prepare(x, 4, stride)
    ref = o.gemm(ocodes, oscales, wt, ws, n, k, residual=res)
    out = cq.project_quantized(to_dev_bf16(x), wdev, residual=to_dev_bf16(res))
    got = from_dev_bf16(out)
    nan_ref = np.isnan(o.bf16_to_f32(ref))
    assert np.array_equal(np.isnan(o.bf16_to_f32(got)), nan_ref)
    assert np.array_equal(got[~nan_ref], ref[~nan_ref])


def test_silu_every_bf16_input(cq):
    """The SwiGLU epilogue's SiLU (approximate exp2 and reciprocal with Ziv's rounding test,
    the table near BF16 rounding midpoints) equals the reference SiLU on all 65,536 BF16 bit
    patterns, NaN payloads included (oracle: swiglu with up = 1, exact for every value)."""
    g = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ones = np.full(65536, 0x3F80, dtype=np.uint16)
    ref = o.swiglu(g, ones)
    got = from_dev_bf16(cq.silu(to_dev_bf16(g)))
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, [(hex(int(i)), hex(int(got[i])), hex(int(ref[i]))) for i in bad[:8]]


@pytest.mark.parametrize("m,n,k", [(1, 256, 2048), (130, 512, 2048), (513, 256, 4096), (77, 768, 6144)])
def test_gemm_swiglu_epilogue(cq, m, n, k):
    """Gate|up in one launch with SwiGLU in the epilogue (clefq_gemm_swiglu_s8, the gate|up step
    of clefq_mlp) equals swiglu of the two oracle projections, bit for bit.  Row 0 is scaled so
    that its projections reach the dense epilogue's finite BF16 clamp and the SwiGLU products
    overflow; NaN positions, if any, must agree."""
    rng = np.random.default_rng(m + n + k)
    _, gt, gs, gdev = _weight(rng, n, k)
    _, ut, us, udev = _weight(rng, n, k)
    x = bf16_normal(rng, (m, k))
    x[0, :] = o.f32_to_bf16(np.full(k, 1e34, np.float32))
    stride = o.stride_for(k)
    _, ocodes, oscales, _ = o.prepare(x, 4, stride)
    ref = o.swiglu(o.gemm(ocodes, oscales, gt, gs, n, k), o.gemm(ocodes, oscales, ut, us, n, k))
    a = cq.prepare(to_dev_bf16(x), 4, stride)
    nan_ref = np.isnan(o.bf16_to_f32(ref))
    for _ in range(2):
        got = from_dev_bf16(cq.project_swiglu_prepared(m, gdev, udev, a))
        assert np.array_equal(np.isnan(o.bf16_to_f32(got)), nan_ref)
        assert np.array_equal(got[~nan_ref], ref[~nan_ref])
    # a wider output row (out_ld > n) leaves the padding untouched
    wide = torch.full((m, n + 256), -1.0, dtype=torch.bfloat16, device="cuda")
    cq.project_swiglu_prepared(m, gdev, udev, a, out=wide[:, :n])
    got = from_dev_bf16(wide)
    assert np.array_equal(got[:, :n][~nan_ref], ref[~nan_ref])
    assert np.all(got[:, n:] == o.f32_to_bf16(np.float32(-1.0)))


def test_gemm_swiglu_rejects_unsupported_shapes(cq):
    rng = np.random.default_rng(3)
    for n, k in ((128, 2048), (256, 1024)):       # n % 256, K below the deep kernel's range
        _, _, _, gdev = _weight(rng, n, k)
        _, _, _, udev = _weight(rng, n, k)
        a = cq.prepare(to_dev_bf16(bf16_normal(rng, (4, k))), 4, o.stride_for(k))
        with pytest.raises(ValueError):
            cq.project_swiglu_prepared(4, gdev, udev, a)


@pytest.mark.parametrize("m,h,inter", [(200, 1024, 768), (300, 2048, 768), (1, 4096, 256), (257, 4096, 1280),
                                        (129, 4096, 512)])
def test_mlp_block(cq, m, h, inter):
    """Dense SwiGLU MLP block through one C-ABI call, bit-exact to the oracle's separate
    steps (prepare, gate, up, swiglu, prepare, down); hidden 4096 with inter a multiple of 256
    takes SwiGLU in the gate|up epilogue, the others SwiGLU in the packing."""
    rng = np.random.default_rng(5 + m)
    ws = []
    for n, k in ((inter, h), (inter, h), (h, inter)):
        _, wt, s, dev = _weight(rng, n, k)
        ws.append(((wt, s, n), dev))
    x = bf16_normal(rng, (m, h))
    ref = o.mlp_block(x, ws[0][0], ws[1][0], ws[2][0])
    for _ in range(2):
        out = cq.mlp(to_dev_bf16(x), ws[0][1], ws[1][1], ws[2][1])
        assert np.array_equal(from_dev_bf16(out), ref)
    cq.status()


@pytest.mark.parametrize("chunk,pinned,residual", [(64, True, False), (77, True, True), (200, False, True),
                                                   (1000, True, False)])
def test_mlp_block_host_chunks(cq, chunk, pinned, residual):
    """Host-to-host MLP (clefq_mlp_host): row chunks streamed through the GPU give the
    oracle's block bit for bit, for chunk sizes that do and do not divide the rows."""
    rng = np.random.default_rng(chunk)
    m, h, inter = 200, 1024, 768
    ws = []
    for n, k in ((inter, h), (inter, h), (h, inter)):
        _, wt, s, dev = _weight(rng, n, k)
        ws.append(((wt, s, n), dev))
    x = bf16_normal(rng, (m, h))
    res = bf16_normal(rng, (m, h)) if residual else None
    if res is None:
        ref = o.mlp_block(x, ws[0][0], ws[1][0], ws[2][0])
    else:  # the oracle's steps with the residual fused into the down projection
        _, xc, xs, _ = o.prepare(x, 4, o.stride_for(h))
        g = o.gemm(xc, xs, *ws[0][0], h)
        u = o.gemm(xc, xs, *ws[1][0], h)
        _, hc, hs, _ = o.prepare(o.swiglu(g, u), 4, o.stride_for(inter))
        ref = o.gemm(hc, hs, *ws[2][0], inter, residual=res)

    def host(a):
        t = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
        return t.pin_memory() if pinned else t
    for _ in range(2):
        out = cq.mlp_host(host(x), ws[0][1], ws[1][1], ws[2][1], residual=None if res is None else host(res),
                          chunk_rows=chunk)
        assert not out.is_cuda
        assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), ref)
    # a stream of calls (each call's input copies overlap the previous call's kernels)
    outs, events = [], []
    for _ in range(3):
        ev = torch.cuda.Event()
        outs.append(cq.mlp_host(host(x), ws[0][1], ws[1][1], ws[2][1], residual=None if res is None else host(res),
                                chunk_rows=chunk, sync=False, streaming=True, done_event=ev))
        events.append(ev)
    for ev, out in zip(events, outs):
        ev.synchronize()
        assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), ref)
    cq.status()


# ---------------------------------------------------------------------------------------
# MoE operators
# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("experts,topk", [(128, 8), (64, 8), (128, 4)])
@pytest.mark.parametrize("phase", [0, 1, 2, 3])
@pytest.mark.parametrize("bf", [0, 1])
def test_route(cq, golden, experts, topk, phase, bf):
    key = f"route_e{experts}_k{topk}_p{phase}_bf{bf}"
    logits = golden[key + "_logits"]
    ref = o.route(logits, topk)
    dev = to_dev_bf16(logits) if bf else to_dev(logits)
    out = cq.omni_route(dev, topk).cpu().numpy()
    assert np.array_equal(out[:, :topk], golden[key + "_ids"])
    assert same_bits_f32(out, ref)


def test_route_random_large(cq):
    rng = np.random.default_rng(11)
    logits = bf16_normal(rng, (4099, 128))
    ref = o.route(logits, 8)
    out = cq.omni_route(to_dev_bf16(logits), 8).cpu().numpy()
    assert same_bits_f32(out, ref)


@pytest.mark.parametrize("tokens", [1, 17, 64, 65, 255, 256, 2048, 5000])
@pytest.mark.parametrize("phase", [0, 1, 2])
def test_group_order_tasks(cq, tokens, phase):
    from tests.golden.make_golden import expert_routes
    routes = expert_routes(tokens, phase == 1, phase)
    g_ref, o_ref = o.group(routes)
    groups, order = cq.omni_group_routes_ordered(to_dev(routes))
    g = groups.cpu().numpy()
    for e in range(128):
        n = int(g_ref[e, 0])
        assert np.array_equal(g[e, : n + 1], g_ref[e, : n + 1])
    assert np.array_equal(order.cpu().numpy(), o_ref)
    tasks = cq.omni_expert_tasks(groups, tokens).cpu().numpy()
    t_ref = o.tasks(g_ref, tokens)
    total = int(t_ref[0])
    assert np.array_equal(tasks[: 1 + 2 * total], t_ref[: 1 + 2 * total])


def _expert_weights(rng, experts, n, k):
    w = bf16_normal(rng, (experts * n, k), 0.05)
    wt, ws = o.pack_weight(w)
    return wt, ws, cq_weight(wt, ws, experts * n, k, 4)


@pytest.mark.parametrize("tokens,skewed", [(1, False), (37, False), (300, True), (1000, False)])
@pytest.mark.parametrize("routed,k,n", [(False, 512, 256), (True, 256, 512), (False, 256, 384), (True, 256, 384),
                                        (True, 768, 512), (False, 768, 256)])
def test_expert_matches_oracle(cq, tokens, skewed, routed, k, n):
    """Grouped INT4 experts, bit-exact (src/benchmarking/omni.rs:176-345 fixtures); n=384
    runs the one-CTA kernel, multiples of 256 the CTA-pair kernels (K <= 768: the
    weight-resident kernel, whose units of one expert's tiles end at ragged expert tails)."""
    from tests.golden.make_golden import expert_routes
    rng = np.random.default_rng(tokens)
    experts, topk = 128, 8
    wt, ws, wdev = _expert_weights(rng, experts, n, k)
    routes = expert_routes(tokens, skewed, 0)
    groups, _ = o.group(routes)
    rows = tokens * topk if routed else tokens
    i = np.arange(rows * k)
    x = o.f32_to_bf16(((i * 17) % 251).astype(np.float32) / 128 - 1).reshape(rows, k)
    _, xc, xs, _ = o.prepare(x, 4, o.stride_for(k))
    ref = o.expert(xc, xs, wt, ws, groups, tokens, k, n, routed)
    a = cq.prepare(to_dev_bf16(x), 4, o.stride_for(k))
    for _ in range(2):
        out = cq.omni_expert(a, to_dev(routes), to_dev(groups), wdev, routed)
        assert np.array_equal(from_dev_bf16(out), ref)


@pytest.mark.parametrize("ordered", [True, False])
@pytest.mark.parametrize("tokens,width", [(1, 2048), (37, 2048), (513, 2048), (37, 264)])
def test_combine(cq, ordered, tokens, width):
    """Top-8 combine, bit-exact: 16 columns per thread when the width is a multiple of 16,
    8 otherwise (width 264)."""
    from tests.golden.make_golden import expert_routes
    rng = np.random.default_rng(tokens)
    routes = expert_routes(tokens, False, 1)
    routes[:, 8:] = o.bf16_to_f32(o.f32_to_bf16(rng.random((tokens, 8)).astype(np.float32)))
    values = bf16_normal(rng, (tokens * 8, width))
    _, order = o.group(routes)
    ref = o.combine(values, routes, order if ordered else None)
    out = cq.omni_combine_ordered(to_dev_bf16(values), to_dev(routes), to_dev(order) if ordered else None)
    assert np.array_equal(from_dev_bf16(out), ref)


@pytest.mark.parametrize("ordered", [True, False])
@pytest.mark.parametrize("topk", [4, 3, 2])
def test_combine_other_topk(cq, ordered, topk):
    """Combine with topk other than 8 (compile-time specialisations for 4 and 2, the generic
    kernel for 3): distinct random experts per token, bit-exact."""
    rng = np.random.default_rng(topk)
    tokens, width, experts = 129, 512, 64
    ids = np.stack([rng.choice(experts, topk, replace=False) for _ in range(tokens)]).astype(np.float32)
    probs = o.bf16_to_f32(o.f32_to_bf16(rng.random((tokens, topk)).astype(np.float32)))
    routes = np.concatenate([ids, probs], axis=1).astype(np.float32)
    values = bf16_normal(rng, (tokens * topk, width))
    _, order = o.group(routes, experts)
    ref = o.combine(values, routes, order if ordered else None)
    out = cq.omni_combine_ordered(to_dev_bf16(values), to_dev(routes), to_dev(order) if ordered else None)
    assert np.array_equal(from_dev_bf16(out), ref)


@pytest.mark.parametrize("tokens", [300, 1024])
def test_moe_block(cq, tokens):
    """The fused MoE block (route -> groups -> gate|up -> SwiGLU packing -> down -> combine)
    equals the oracle's separate reference operators bit for bit."""
    rng = np.random.default_rng(tokens)
    experts, topk, hidden, inter = 128, 8, 512, 256
    gt, gs, gdev = _expert_weights(rng, experts, inter, hidden)
    ut, us, udev = _expert_weights(rng, experts, inter, hidden)
    dt, ds, ddev = _expert_weights(rng, experts, hidden, inter)
    x = bf16_normal(rng, (tokens, hidden))
    logits = bf16_normal(rng, (tokens, experts))
    ref, ref_routes, _, _ = o.moe_layer(x, logits, (gt, gs, inter), (ut, us, inter), (dt, ds, hidden))
    routes_out = torch.empty((tokens, 2 * topk), dtype=torch.float32, device="cuda")
    for _ in range(2):
        out = cq.omni_moe(to_dev_bf16(x), to_dev_bf16(logits), gdev, udev, ddev, routes_out=routes_out)
        assert same_bits_f32(routes_out.cpu().numpy(), ref_routes)
        assert np.array_equal(from_dev_bf16(out), ref)
    cq.status()


def test_calls_from_threads_on_own_streams(cq):
    """The C ABI is reentrant on different streams: four host threads, each on its own CUDA
    stream, run projections of different shapes (two-sub-tile, one-sub-tile and one-CTA GEMM
    kernels, int4 and int8) at the same time; every result equals the oracle."""
    import threading
    cases = [(400, 512, 1024, 4), (37, 256, 512, 4), (65, 128, 2048, 4), (200, 256, 1024, 8)]
    prepared = []
    for m, n, k, bits in cases:
        rng = np.random.default_rng(m * 7 + n + bits)
        _, wt, ws, wdev = _weight(rng, n, k, bits)
        x = bf16_normal(rng, (m, k))
        _, ocodes, oscales, _ = o.prepare(x, bits, o.stride_for(k, bits))
        prepared.append((x, wdev, bits, o.gemm(ocodes, oscales, wt, ws, n, k, bits=bits)))
    results = [None] * len(cases)
    errors = []

    def work(i):
        try:
            x, wdev, bits, _ = prepared[i]
            stream = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                xd = to_dev_bf16(x)
                outs = [cq.project_quantized(xd, wdev) for _ in range(5)]
            stream.synchronize()
            results[i] = [from_dev_bf16(t) for t in outs]
        except Exception as e:  # reported on the main thread
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(cases))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for (_, _, _, ref), outs in zip(prepared, results):
        for got in outs:
            assert np.array_equal(got, ref)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,k,n,padded", [(33, 1024, 256, True), (7, 512, 128, False), (65, 2048, 384, True)])
@pytest.mark.parametrize("varying", [False, True])
def test_gemm_exact_benchmark_inputs(cq, bits, m, k, n, padded, varying):
    """The reference's packed integer GEMM benchmark fixture (src/benchmarking.rs:190-197,
    286-410) through clefq_gemm: raw codes (int4 codes include -8, which prepared rows never
    hold), uniform or varying row scales with zero rows; bit-exact to the oracle."""
    from tests.test_oracle_golden import _bench_codes, _bench_scales
    stride = k + (512 // bits if padded and k % 1024 == 0 else 0)
    _, a_words = _bench_codes(m, k, bits, stride)
    _, w_words = _bench_codes(n, k, bits, stride)
    a_s = _bench_scales(m, bits, 3, 17, varying)
    w_s = _bench_scales(n, bits, 7, 23, varying)
    w_tiled = o.retile(w_words, n, k, bits)
    ref = o.gemm(a_words, a_s, w_tiled, w_s, n, k, bits=bits)
    words = stride // (32 // bits)
    storage = to_dev(np.concatenate([a_words.ravel().view(np.int32), a_s.view(np.int32)]))
    a = cq.Prepared(storage, storage[: m * words].view(m, words), storage[m * words:].view(torch.float32), None, None,
                    bits, stride)
    wdev = cq.QuantizedWeight(to_dev(w_tiled.view(np.int32)), to_dev(w_s), n, k, stride, bits)
    for _ in range(2):
        out = cq.project_prepared(m, wdev, a)
        assert np.array_equal(from_dev_bf16(out), ref)
