"""Pin the CPU oracle to the reference's own test oracles and known answers (no GPU).

Golden vectors come from tests/golden/make_golden.py, an independent numpy restatement of
the reference's in-test CPU oracles; the cases below mirror the reference tests named in
each docstring.
"""
import numpy as np
import pytest

from oracle import oracle as o


def _logical(codes, width, bits):
    return codes[:, : width // (32 // bits)]


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("width", [256, 768, 1280, 5120, 6144, 8192, 17408])
def test_rotated_packing_matches_golden(golden, bits, width):
    """src/quantized.rs:1072-1129 rotated_packing_cpu_oracle: exact codes, scales 1e-6."""
    key = f"pack_b{bits}_w{width}"
    x = golden[key + "_x"]
    stride = width + 512 // bits
    storage, codes, scales, _ = o.prepare(x, bits, stride)
    assert np.array_equal(_logical(codes, width, bits), golden[key + "_words"])
    exp = golden[key + "_scales"]
    assert np.all(np.abs(scales - exp) <= exp * 1e-6)
    # storage layout: codes[rows][stride/P] then f32 scales (src/quantized.rs:656-664)
    words = stride // (32 // bits)
    assert storage.size == 3 * (words + 1)
    assert np.array_equal(storage[3 * words:].view(np.float32), scales)


@pytest.mark.parametrize("bits", [4, 8])
def test_exceptional_rows_match_golden(golden, bits):
    """src/quantized.rs:1131-1185: NaN / Inf / bf16 MAX rows get an inf scale and zero codes;
    subnormal rows keep the 1e-30 floor."""
    x = golden[f"exc_b{bits}_x"]
    _, codes, scales, _ = o.prepare(x, bits, 5120 + 512 // bits)
    assert np.array_equal(_logical(codes, 5120, bits), golden[f"exc_b{bits}_words"])
    assert np.array_equal(scales.view(np.uint32), golden[f"exc_b{bits}_scales"].view(np.uint32))
    assert np.isinf(scales[3]) and np.isinf(scales[4]) and np.isinf(scales[5])
    assert not np.any(_logical(codes, 5120, bits)[3:6])


def test_rotation_preserves_inner_product():
    """src/quantized.rs:857-876: <Ha, Hb>/256 == <a, b> within 1e-8 (f64 sums)."""
    i = np.arange(512)
    a = o.f32_to_bf16(((i * 17 % 71).astype(np.float32) - 35) / 64)
    b = o.f32_to_bf16(((i * 31 % 59).astype(np.float32) - 29) / 64)
    expected = float(np.dot(o.bf16_to_f32(a).astype(np.float64), o.bf16_to_f32(b).astype(np.float64)))
    # Recover the rotation from prepare: with 8-bit codes the rotated values are the codes
    # scaled back, too coarse here; so compare through the golden numpy rotation instead.
    from tests.golden.make_golden import rotated
    actual = float(np.dot(rotated(a).astype(np.float64), rotated(b).astype(np.float64)) / 256)
    assert abs(actual - expected) < 1e-8


@pytest.mark.parametrize("bits,rows,cols,padded", [(4, 256, 1024, True), (4, 384, 512, False),
                                                  (8, 128, 256, False)])
def test_retile_block_formula(bits, rows, cols, padded):
    """src/quantized.rs:1369-1407 retiled_codes_match_block_formula."""
    stride = cols + (512 // bits if padded else 0)
    in_words, words = stride // (32 // bits), cols // (32 // bits)
    values = (np.arange(rows * in_words, dtype=np.uint64) * 2654435761 % (1 << 32)).astype(np.uint32)
    tiled = o.retile(values.reshape(rows, in_words), rows, cols, bits)
    assert tiled.size == rows * words
    n, q = np.meshgrid(np.arange(rows), np.arange(words), indexing="ij")
    at = ((n // 128) * (words // 32) + q // 32) * 4096 + (n % 128) * 32 + q % 32
    assert np.array_equal(tiled[at], values.reshape(rows, in_words)[:, :words])


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("index", [0, 1])
@pytest.mark.parametrize("rows", [1, 17])
@pytest.mark.parametrize("start", [0, 1])
def test_gemm_matches_integer_dot(golden, bits, index, rows, start):
    """src/quantized.rs:977-1070: int32 accumulators exact; bf16 output within
    max(|a|,|e|)/128 + 1e-6 of bf16(dot * a_scale * w_scale)."""
    key = f"gemm_b{bits}_i{index}_r{rows}_s{start}"
    w = golden[f"gemm_b{bits}_i{index}_w"]
    wt, ws = o.pack_weight(w, bits)
    _, codes, scales, _ = o.prepare(golden[key + "_x"], bits, 256)
    out, acc = o.gemm(codes, scales, wt, ws, 256, 256, bits=bits, want_acc=True)
    assert np.array_equal(acc, golden[key + "_dot"])
    actual = o.bf16_to_f32(out)
    expected = golden[key + "_expected"]
    assert np.all(np.isfinite(actual))
    tol = np.maximum(np.abs(actual), np.abs(expected)) / 128 + 1e-6
    assert np.all(np.abs(actual - expected) <= tol)


@pytest.mark.parametrize("experts,topk", [(128, 8), (64, 8), (128, 4)])
@pytest.mark.parametrize("phase", [0, 1, 2, 3])
@pytest.mark.parametrize("bf", [0, 1])
def test_router_matches_serial_spec(golden, experts, topk, phase, bf):
    """src/benchmarking/omni.rs:6-102: ids equal the serial scan exactly (ties and +-0 go
    to the lowest id); probabilities within one bf16 step (exp bits are unpinned)."""
    key = f"route_e{experts}_k{topk}_p{phase}_bf{bf}"
    routes = o.route(golden[key + "_logits"], topk)
    assert np.array_equal(routes[:, :topk], golden[key + "_ids"])
    p, e = routes[:, topk:], golden[key + "_probs"]
    assert np.all(np.abs(p - e) <= np.maximum(np.abs(e), 1e-30) / 128)


@pytest.mark.parametrize("tokens", [1, 17, 64, 65, 128, 255, 256])
@pytest.mark.parametrize("phase", [0, 1, 2])
def test_grouping_order_tasks(golden, tokens, phase):
    """src/omni.rs:906-942 (stable groups), src/benchmarking/omni.rs:277-303 (tasks) and
    :425-437 (ascending expert order)."""
    key = f"group_t{tokens}_p{phase}"
    groups, order = o.group(golden[key + "_routes"])
    exp_groups = golden[key + "_groups"]
    for e in range(128):
        n = int(exp_groups[e, 0])
        assert np.array_equal(groups[e, : n + 1], exp_groups[e, : n + 1])
    assert np.array_equal(order, golden[key + "_order"])
    tasks = o.tasks(groups, tokens)
    exp_tasks = golden[key + "_tasks"]
    total = int(exp_tasks[0])
    assert np.array_equal(tasks[: 1 + 2 * total], exp_tasks[: 1 + 2 * total])


def test_combine_ordered_equals_unordered():
    """src/benchmarking/omni.rs:360-442: the ordered combine is bit-identical to the
    ascending-expert scan."""
    from tests.golden.make_golden import expert_routes
    tokens, width = 37, 256
    for phase in range(3):
        routes = expert_routes(tokens, phase == 1, phase)
        for t in range(tokens):
            for r in range(8):
                routes[t, 8 + r] = o.bf16_to_f32(o.f32_to_bf16(np.float32(((r + phase) % 8 + 1) / 36)))[()]
        i = np.arange(tokens * 8 * width)
        values = o.f32_to_bf16(((i * 17 + phase * 7) % 251).astype(np.float32) / 128 - 1).reshape(tokens * 8, width)
        _, order = o.group(routes)
        a = o.combine(values, routes, order)
        b = o.combine(values, routes, None)
        assert np.array_equal(a, b)
        assert np.all(np.isfinite(o.bf16_to_f32(a)))


def test_routed_experts_match_sparse_oracle():
    """src/omni.rs:944-1051: route -> expert(up) -> expert(up, routed) -> combine against
    the closed-form sparse answer, INT4 tolerance 0.08."""
    experts, topk = 128, 8
    i = np.arange(3 * experts)
    logits = o.f32_to_bf16(((i * 37 + i // experts * 11) % experts).astype(np.float32) / 16).reshape(3, experts)
    j = np.arange(3 * 256)
    x = o.f32_to_bf16((j % 17).astype(np.float32) / 16 - 0.5).reshape(3, 256)
    rows = np.arange(experts * 256)
    w = np.zeros((experts * 256, 256), dtype=np.float32)
    w[rows, rows % 256] = (rows // 256 + 1).astype(np.float32) / 128
    wt, ws = o.pack_weight(o.f32_to_bf16(w))
    routes = o.route(logits, topk)
    groups, _ = o.group(routes)
    _, xc, xs, _ = o.prepare(x, 4, 256)
    v1 = o.expert(xc, xs, wt, ws, groups, 3, 256, 256, False)
    _, vc, vs, _ = o.prepare(v1, 4, 256)
    v2 = o.expert(vc, vs, wt, ws, groups, 3, 256, 256, True)
    out = o.bf16_to_f32(o.combine(v2, routes, None))
    lf = o.bf16_to_f32(logits)
    xf = o.bf16_to_f32(x)
    for t in range(3):
        ranked = sorted(range(experts), key=lambda e: -lf[t, e])
        assert [int(q) for q in routes[t, :topk]] == ranked[:topk]
        mx = lf[t, ranked[0]]
        sel = [(e, np.float32(np.exp(np.float32(lf[t, e] - mx)))) for e in ranked[:topk]]
        s = np.float32(sum(p for _, p in sel))
        sel = sorted([(e, o.bf16_to_f32(o.f32_to_bf16(np.float32(p / s)))) for e, p in sel])
        for c in range(256):
            expected = np.float32(0)
            for e, p in sel:
                y = o.bf16_to_f32(o.f32_to_bf16(np.float32(xf[t, c] * (e + 1) / 128)))
                y = o.bf16_to_f32(o.f32_to_bf16(np.float32(y * (e + 1) / 128)))
                y = o.bf16_to_f32(o.f32_to_bf16(np.float32(y * p)))
                expected = o.bf16_to_f32(o.f32_to_bf16(np.float32(expected + y)))
            assert abs(out[t, c] - expected) <= 0.08


def test_swiglu_within_one_bf16_step():
    """src/ops.rs:482-525 semantics bf16(bf16(silu(g)) * u); exp bits unpinned, so compare
    to a float64-exp restatement within one bf16 step."""
    i = np.arange(8 * 768)
    g = o.f32_to_bf16(((i * 17 % 1031).astype(np.float32) - 515) / 16)
    u = o.f32_to_bf16(((i * 29 % 997).astype(np.float32) - 498) / 32)
    out = o.bf16_to_f32(o.swiglu(g, u))
    gf, uf = o.bf16_to_f32(g).astype(np.float64), o.bf16_to_f32(u)
    act = o.bf16_to_f32(o.f32_to_bf16((gf / (1 + np.exp(-gf))).astype(np.float32)))
    exp = o.bf16_to_f32(o.f32_to_bf16(act * uf))
    assert np.all(np.abs(out - exp) <= np.abs(exp) / 128 + 1e-30)


def test_exp_error_bound():
    """The shared exp (Cody-Waite + degree-7 Taylor) stays within 2 ulp of float64 exp."""
    x = np.concatenate([np.linspace(-103, 88.7, 200001, dtype=np.float32),
                        np.array([0.0, -0.0, 1e-8, -1e-8], np.float32)])
    got = o.exp(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    normal = ref > 1.2e-38
    ulp = np.spacing(ref[normal].astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got[normal] - ref[normal]) / ulp) <= 2.0
    assert np.isinf(o.exp(np.array([89.0], np.float32))[0])
    assert o.exp(np.array([-104.0], np.float32))[0] == 0
    assert np.isnan(o.exp(np.array([np.nan], np.float32))[0])


def _norm_case_values(rows, width):
    """The input rows of src/quantized.rs:1553-1774: a (rows + 2) x width array whose row
    class (i / width) % 11 selects signed zeros, tiny, BF16 MAX, subnormal, huge, NaN/+Inf/-Inf
    at one column, +-1 or scaled ramp values; the packed rows are 1 .. rows."""
    i = np.arange((rows + 2) * width, dtype=np.int64)
    c, cls = i % width, (i // width) % 11
    value = ((i * 37 % 1031).astype(np.float32) - np.float32(515)) / np.float32(37)
    v = value.copy()
    v[cls == 0] = np.where(c[cls == 0] % 2 == 0, np.float32(0.0), np.float32(-0.0))
    v[cls == 1] = value[cls == 1] * np.float32(1e-5)
    v[cls == 2] = o.bf16_to_f32(np.uint16(0x7F7F))
    v[cls == 3] = o.bf16_to_f32(np.uint16(1))
    v[cls == 4] = value[cls == 4] * np.float32(1e15)
    v[(cls == 5) & (c == 37)] = np.nan
    v[(cls == 6) & (c == 113)] = np.inf
    v[(cls == 7) & (c == 259)] = -np.inf
    v[cls == 8] = np.where(c[cls == 8] % 2 == 0, np.float32(1.0), np.float32(-1.0))
    v[cls == 9] = value[cls == 9] * np.float32(1e-3)
    return o.f32_to_bf16(v.astype(np.float32)).reshape(rows + 2, width)


def _norm_case_weight(width, exceptional):
    i = np.arange(3 * width, dtype=np.int64)
    if exceptional:
        w = np.full(i.shape, 0.5, np.float32)
        w[i % 1009 == 0] = np.nan
        w[i % 1009 == 1] = np.inf
        w[i % 1009 == 2] = -np.inf
        w[i % 1009 == 3] = o.bf16_to_f32(np.uint16(0x7F7F))
    else:
        w = ((i * 13 % 127).astype(np.float32) - np.float32(63)) / np.float32(128)
        w[i % 19 == 0] = -1.0
        w[i % 19 == 1] = -0.0
        w[i % 19 == 2] = 0.0
    return o.f32_to_bf16(w.astype(np.float32))[2 * width:]


def _bf16_ulp(a, b):
    def ordered(h):
        h = h.astype(np.int64)
        return np.where(h & 0x8000, (~h) & 0xFFFF, h | 0x8000)
    return np.abs(ordered(a) - ordered(b))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("exceptional_weight", [False, True])
@pytest.mark.parametrize("rows", [1, 7, 65, 158])
def test_norm_packing_known_answers(bits, exceptional_weight, rows):
    """src/quantized.rs:1553-1774 on the oracle (width 5120): packing with the RMSNorm stored
    gives the same codes and scales as without storing; packing the stored normalised rows
    separately stays within the reference's bounds of the fused codes (|delta| <= 1 on at most
    1% of codes, scales within 0.4%; here they are equal, since the fused packing quantises the
    BF16 normalised values); and on finite rows without subnormal inputs every normalised value
    is within one BF16 step of the reference's FP64 RMS oracle."""
    width = 5120
    values = _norm_case_values(rows, width)
    x = values[1:rows + 1]
    w = _norm_case_weight(width, exceptional_weight)
    stride = width + 512 // bits
    fused, fcodes, fscales, _ = o.prepare(x, bits, stride, o.NORM, w)
    stored, _, sscales, norm = o.prepare(x, bits, stride, o.NORM_STORE, w)
    assert np.array_equal(fused, stored)
    _, ucodes, uscales, _ = o.prepare(norm, bits, stride)
    p = 32 // bits
    for lane in range(p):
        def dec(words):
            return ((words[:, : width // p] << np.uint32(32 - bits * (lane + 1))).view(np.int32)
                    >> np.int32(32 - bits))
        assert np.abs(dec(fcodes) - dec(ucodes)).max() <= 1
    assert np.array_equal(_logical(fcodes, width, bits), _logical(ucodes, width, bits))
    finite = np.isfinite(uscales)
    assert np.array_equal(fscales[~finite].view(np.uint32), uscales[~finite].view(np.uint32))
    assert np.all(np.abs(fscales[finite] - uscales[finite]) <= np.maximum(np.abs(uscales[finite]), 1e-30) * 0.004)
    if exceptional_weight:
        return
    wf = (o.bf16_to_f32(w) + np.float32(1.0)).astype(np.float64)
    checked = 0
    for row in sorted({0, rows // 2, rows - 1}):
        v = o.bf16_to_f32(x[row])
        if not (np.all(np.isfinite(v)) and np.all(np.abs(v) <= 1e16)
                and np.all((v == 0) | (np.abs(v) >= np.finfo(np.float32).tiny))):
            continue
        vd = v.astype(np.float64)
        inv = 1.0 / np.sqrt(np.sum(vd * vd) / width + np.float64(np.float32(1e-6)))
        ref = o.f32_to_bf16((vd * inv * wf).astype(np.float32))
        assert _bf16_ulp(norm[row], ref).max() <= 1, row
        checked += 1
    assert rows < 7 or checked > 0


def _bench_codes(rows, k, bits, stride):
    """The packed integer GEMM fixture of src/benchmarking.rs:190-197,351-364: element i of a
    row-major rows x k matrix is gemm_value(i) = ((i * 17 % 251) - 125) / 128, for int4 rounded
    (half away from zero, as Rust's round) to eighths in [-8, 7] / 8; divided by the uniform
    scale it is an exact code, packed little-endian, code c at bits (c % P) * bits of word c / P.
    Returns (codes as int64, packed words [rows][stride / P])."""
    i = np.arange(rows * k, dtype=np.int64).reshape(rows, k)
    value = ((i * 17 % 251).astype(np.float32) - np.float32(125)) / np.float32(128)
    if bits == 4:
        t = value * np.float32(8)
        code = np.clip(np.sign(t) * np.floor(np.abs(t) + np.float32(0.5)), -8, 7).astype(np.int64)
    else:
        code = (value * np.float32(128)).astype(np.int64)
    p = 32 // bits
    nib = (code & ((1 << bits) - 1)).astype(np.uint64).reshape(rows, k // p, p)
    words = np.zeros((rows, stride // p), np.uint32)
    words[:, : k // p] = (nib << (np.arange(p, dtype=np.uint64) * bits)).sum(axis=2).astype(np.uint32)
    return code, words


def _bench_scales(rows, bits, factor, zero_period, varying):
    if not varying:
        return np.full(rows, 1.0 / (1 << (bits - 1)), np.float32)
    r = np.arange(rows, dtype=np.int64)
    s = ((r * factor % 31 + 1).astype(np.float32) / np.float32(257.0)) * np.exp2(
        -((r * factor % 5) * 4).astype(np.float32))
    s[r % zero_period == 0] = 0.0
    return s.astype(np.float32)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,k,n,padded", [(33, 1024, 256, True), (7, 512, 128, False), (65, 2048, 384, True)])
@pytest.mark.parametrize("varying", [False, True])
def test_gemm_exact_benchmark_inputs(bits, m, k, n, padded, varying):
    """The reference's packed integer GEMM benchmark inputs (src/benchmarking.rs:286-410):
    codes that are exact (int4 codes include -8), uniform scales 1/8 or 1/128, or the
    CLEF_BENCH_INTEGER_ROW_SCALES variant (zero rows, scales down to 2^-16).  The oracle's int32
    accumulators equal the exact integer dot, and its BF16 outputs equal the epilogue
    (f32(acc) * ws) * as rounded once; with uniform scales the product before rounding is
    exact."""
    stride = k + (512 // bits if padded and k % 1024 == 0 else 0)
    a_code, a_words = _bench_codes(m, k, bits, stride)
    w_code, w_words = _bench_codes(n, k, bits, stride)
    a_s = _bench_scales(m, bits, 3, 17, varying)
    w_s = _bench_scales(n, bits, 7, 23, varying)
    w_tiled = o.retile(w_words, n, k, bits)
    out, acc = o.gemm(a_words, a_s, w_tiled, w_s, n, k, bits=bits, want_acc=True)
    exact = a_code @ w_code.T
    assert np.array_equal(acc.astype(np.int64), exact)
    y = (exact.astype(np.float32) * w_s[None, :]) * a_s[:, None] + np.float32(0.0)
    big = o.bf16_to_f32(np.uint16(0x7F7F))
    y = np.where(np.isfinite(y), np.clip(y, -big, big), y).astype(np.float32)
    assert np.array_equal(out, o.f32_to_bf16(y))
    if not varying:
        assert np.array_equal(y.astype(np.float64), exact.astype(np.float64) * (a_s[0] * np.float64(w_s[0])))


def _swiglu_case(rows, width):
    """The gate and up rows of src/quantized.rs:1187-1266: gate row class (i / width) % 7 gives
    zeros, one NaN (column 259), one +Inf (column 515), BF16 MAX, a BF16 subnormal, +-80, or a
    ramp; up is a ramp; the packed rows are gate rows 1 .. rows and up rows 2 .. rows + 1."""
    i = np.arange((rows + 2) * width, dtype=np.int64)
    col, cls = i % width, (i // width) % 7
    g = ((i * 17 % 1031).astype(np.float32) - np.float32(515)) / np.float32(16)
    g[cls == 0] = 0.0
    g[(cls == 1) & (col == 259)] = np.nan
    g[(cls == 2) & (col == 515)] = np.inf
    g[cls == 3] = o.bf16_to_f32(np.uint16(0x7F7F))
    g[cls == 4] = np.uint32(0x00010000).view(np.float32)
    g[cls == 5] = np.where(col[cls == 5] % 2 == 0, np.float32(-80.0), np.float32(80.0))
    j = np.arange((rows + 3) * width, dtype=np.int64)
    u = ((j * 29 % 997).astype(np.float32) - np.float32(498)) / np.float32(32)
    gate = o.f32_to_bf16(g.astype(np.float32)).reshape(rows + 2, width)[1:rows + 1]
    up = o.f32_to_bf16(u.astype(np.float32)).reshape(rows + 3, width)[2:rows + 2]
    return np.ascontiguousarray(gate), np.ascontiguousarray(up)


@pytest.mark.parametrize("width,bits,rows", [(17408, 4, 1), (17408, 4, 158), (17408, 8, 128), (17408, 8, 620),
                                             (768, 4, 8), (768, 4, 136), (768, 4, 2048), (768, 4, 16384)])
def test_fused_swiglu_packing_equals_separate(width, bits, rows):
    """src/quantized.rs:1187-1266: packing with SwiGLU fused in gives the same code words and
    scale bits as SwiGLU followed by plain packing, on the reference's exceptional rows."""
    gate, up = _swiglu_case(rows, width)
    stride = width + 512 // bits
    _, fcodes, fscales, _ = o.prepare(gate, bits, stride, o.SWIGLU, up)
    _, scodes, sscales, _ = o.prepare(o.swiglu(gate, up), bits, stride)
    assert np.array_equal(_logical(fcodes, width, bits), _logical(scodes, width, bits))
    assert np.array_equal(fscales.view(np.uint32), sscales.view(np.uint32))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("rows", [1, 128, 158, 620])
def test_attention_gate_packing_equals_separate(bits, rows):
    """src/quantized.rs:1268-1368 (width 6144, 24 heads): packing with the sigmoid attention
    gate fused in equals the separate steps -- gate columns 512h + 256 .. 512h + 511 of the
    q|gate rows, s = bf16(1 / (1 + exp(-g))), v = bf16(a * s), plain packing -- bit for bit,
    while every Q half of the q|gate rows is NaN and must not be read."""
    width = 6144
    i = np.arange((rows + 2) * width, dtype=np.int64)
    cls = (i // width) % 7
    a = ((i * 29 % 997).astype(np.float32) - np.float32(498)) / np.float32(32)
    a[cls == 0] = 0.0
    a[cls == 3] = o.bf16_to_f32(np.uint16(0x7F7F))
    attn = o.f32_to_bf16(a).reshape(rows + 2, width)[1:rows + 1].copy()
    j = np.arange((rows + 3) * width * 2, dtype=np.int64)
    col, qc = j % (2 * width), (j // (2 * width)) % 7
    q = ((j * 17 % 1031).astype(np.float32) - np.float32(515)) / np.float32(16)
    q[qc == 0] = 0.0
    q[(qc == 1) & (col == 771)] = np.nan
    q[(qc == 2) & (col == 1283)] = np.inf
    q[qc == 3] = o.bf16_to_f32(np.uint16(0x7F7F))
    q[qc == 4] = np.uint32(0x00010000).view(np.float32)
    q[qc == 5] = np.where(col[qc == 5] % 2 == 0, np.float32(-80.0), np.float32(80.0))
    q[col % 512 < 256] = np.nan
    q_gate = o.f32_to_bf16(q.astype(np.float32)).reshape(rows + 3, 2 * width)[2:rows + 2].copy()
    stride = width + 512 // bits
    _, fcodes, fscales, _ = o.prepare(attn, bits, stride, o.ATTN_GATE, q_gate)
    gate = o.bf16_to_f32(q_gate.reshape(rows, 24, 512)[:, :, 256:].reshape(rows, width))
    with np.errstate(all="ignore"):
        s = o.f32_to_bf16(np.float32(1.0) / (np.float32(1.0) + o.exp(-gate).astype(np.float32)))
        v = o.f32_to_bf16(o.bf16_to_f32(attn) * o.bf16_to_f32(s))
    _, scodes, sscales, _ = o.prepare(v, bits, stride)
    assert np.array_equal(_logical(fcodes, width, bits), _logical(scodes, width, bits))
    assert np.array_equal(fscales.view(np.uint32), sscales.view(np.uint32))


@pytest.mark.parametrize("k,rows", [(6144, 127), (6144, 129), (6144, 257), (17408, 129)])
def test_residual_projection_equals_separate_addition(k, rows):
    """src/quantized.rs:1409-1552 (n 5120): the residual-fused projection equals the plain
    projection followed by bf16(residual + y), bit for bit (NaN as NaN), with zero and 1e34
    weight scales, zero activation scales and NaN/Inf/MAX/-0/subnormal residuals."""
    n = 5120
    stride = k + (128 if k % 1024 == 0 else 0)
    words = stride // 8

    def packed(r):
        row = np.arange(r, dtype=np.int64)[:, None, None]
        word = np.arange(k // 8, dtype=np.int64)[None, :, None]
        lane = np.arange(8, dtype=np.int64)[None, None, :]
        code = (row * 17 + word * 7 + lane * 3) % 15 - 7
        data = np.zeros((r, words), np.uint32)
        data[:, : k // 8] = ((code & 15).astype(np.uint64) << (lane.astype(np.uint64) * 4)).sum(axis=2)
        return data

    w_codes = packed(n + 1)[1:]
    i = np.arange(n + 3)
    ws = np.where(i % 23 == 0, 0.0, np.where(i % 29 == 0, 1e34, (i % 31 + 1) / 257.0)).astype(np.float32)[3:]
    a_codes = packed(rows + 2)[2:]
    i = np.arange(rows + 2)
    a_s = np.where(i % 17 == 0, 0.0, (i % 19 + 1) / 131.0).astype(np.float32)[2:]
    i = np.arange((rows + 1) * n, dtype=np.int64)
    r = ((i * 43 % 997).astype(np.float32) - np.float32(498)) / np.float32(257)
    big = o.bf16_to_f32(np.uint16(0x7F7F))
    for idx, val in enumerate([np.nan, np.inf, -np.inf, big, -big, -0.0, 0.0, o.bf16_to_f32(np.uint16(1))]):
        r[i % 1009 == idx] = val
    residual = o.f32_to_bf16(r.astype(np.float32)).reshape(rows + 1, n)[1:].copy()
    w_tiled = o.retile(w_codes, n, k, 4)
    plain = o.gemm(a_codes, a_s, w_tiled, ws, n, k)
    fused = o.gemm(a_codes, a_s, w_tiled, ws, n, k, residual=residual)
    with np.errstate(all="ignore"):
        expected = o.f32_to_bf16(o.bf16_to_f32(residual) + o.bf16_to_f32(plain))
    nan = np.isnan(o.bf16_to_f32(expected))
    assert np.array_equal(np.isnan(o.bf16_to_f32(fused)), nan)
    assert np.array_equal(fused[~nan], expected[~nan])
    # the 1e34 weight scales reach huge outputs (and inf * 0 = NaN where they overflow on a row
    # whose activation scale is zero, as the epilogue order (acc * ws) * as gives)
    pf = o.bf16_to_f32(plain)
    assert np.nanmax(np.abs(pf)) > 1e35 and (pf == 0).any()


def test_golden_file_regenerates_from_its_script(golden):
    """tests/golden/golden.npz is exactly what tests/golden/make_golden.py produces: every
    array, regenerated in memory, equals the committed one (dtype, shape and bits)."""
    from tests.golden import make_golden as mg
    out = {}
    with np.errstate(all="ignore"):
        for cases in (mg.packing_cases, mg.exceptional_cases, mg.gemm_cases, mg.route_cases, mg.group_cases):
            cases(out)
    assert sorted(out) == sorted(golden)
    for name, arr in out.items():
        ref = golden[name]
        arr = np.asarray(arr)
        assert arr.dtype == ref.dtype and arr.shape == ref.shape, name
        assert arr.tobytes() == ref.tobytes(), name
