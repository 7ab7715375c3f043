"""Generate tests/golden/golden.npz -- golden vectors for the INT4 path.

The reference (clef-hrx) cannot run in this image: it needs cargo, the un-vendored
`hrx-rs =0.11.0` crate and an AMD gfx1151 GPU.  Its tests for this path hold no stored
vectors either; they generate inputs from closed-form formulas and check the GPU against
CPU oracles written inside the Rust tests.  This script restates those in-test oracles in
numpy, independently of oracle/clefq_oracle.c, on the same formula inputs, and stores the
inputs and expected outputs:

  pack_*      src/quantized.rs:1072-1129  rotated_packing_cpu_oracle  (rotated(): :801-824,
              quantizer :1000-1015); exact codes, scales to 1e-6 relative
  exc_*       src/quantized.rs:1131-1185  exceptional rows (NaN, Inf, bf16 MAX, subnormal);
              semantics of kernels/prepare_integer.loom:218-291 (non-finite -> inf scale,
              zero codes)
  gemm_*      src/quantized.rs:977-1070   packed_weights_survive_plan_reset: integer dot
              exact, bf16(dot * a_scale * w_scale) within max(|a|,|e|)/128 + 1e-6
  route_*     src/benchmarking/omni.rs:6-102  router phases (ties, +-0, large), serial scan
              of benches/kernels/omni_route_serial.loom; ids exact, probabilities computed
              with a float64 exp (the reference's exp<afn> bits are unpinned)
  group_*     src/omni.rs:906-942  grouped_routes_match_cpu (empty, full, concentrated)
  order_*     src/benchmarking/omni.rs:360-442 ascending-expert order (stable total_cmp sort)

Run:  python tests/golden/make_golden.py      (writes golden.npz next to this file)
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F32 = np.float32


def bf16_bits(x) -> np.ndarray:
    """half::bf16::from_f32: round to nearest even; NaN -> quiet NaN."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    return np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, r).astype(np.uint16)


def bf16_f32(h) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def rotated(row_bf16: np.ndarray) -> np.ndarray:
    """src/quantized.rs:801-824, element by element in float32."""
    out = bf16_f32(row_bf16).astype(F32).copy()
    for g0 in range(0, out.size, 256):
        g = out[g0:g0 + 256]
        for stride in (1, 4, 16, 64):
            for base in range(0, 256, 4 * stride):
                i = np.arange(stride)
                j = base + i
                a, b, c, d = g[j].copy(), g[j + stride].copy(), g[j + 2 * stride].copy(), g[j + 3 * stride].copy()
                s01, s23, d01, d23 = a + b, c + d, a - b, c - d
                g[j] = s01 + d23
                g[j + stride] = s01 - d23
                g[j + 2 * stride] = d01 + s23
                g[j + 3 * stride] = s23 - d01
    return out


def quantize(rot: np.ndarray, bits: int):
    """kernels/prepare_integer.loom:218-291 (== src/quantized.rs:1000-1015 for finite rows)."""
    qmax = F32(127.0 if bits == 8 else 7.0)
    mag = np.abs(rot)
    mag = np.where(mag < np.inf, mag, F32(np.inf))
    m = F32(0.0) if mag.size == 0 else F32(np.max(mag))
    scale = F32(F32(max(F32(m * F32(0.0625)), F32(1e-30))) / qmax)
    if not scale < np.inf:
        return np.zeros(rot.size, dtype=np.int32), scale
    inv = F32(F32(0.0625) / scale)
    codes = np.clip(np.rint((rot * inv).astype(F32)), -qmax, qmax).astype(np.int32)
    return codes, scale


def pack_words(codes: np.ndarray, bits: int) -> np.ndarray:
    p = 32 // bits
    mask = (1 << bits) - 1
    c = (codes.astype(np.int64) & mask).reshape(-1, p).astype(np.uint64)
    shifts = (np.arange(p, dtype=np.uint64) * bits)
    return np.bitwise_or.reduce(c << shifts, axis=1).astype(np.uint32)


def packing_cases(out: dict):
    for bits in (4, 8):
        for width in (256, 768, 1280, 5120, 6144, 8192, 17408):
            vals = np.zeros((3, width), dtype=F32)
            vals[1, 0] = 1.0
            i = np.arange(width)
            vals[2] = ((i * 37 % 257).astype(F32) - F32(128.0)) / F32(91.0)
            x = bf16_bits(vals)
            words, scales = [], []
            for r in range(3):
                codes, s = quantize(rotated(x[r]), bits)
                words.append(pack_words(codes, bits))
                scales.append(s)
            key = f"pack_b{bits}_w{width}"
            out[key + "_x"] = x
            out[key + "_words"] = np.stack(words)
            out[key + "_scales"] = np.array(scales, dtype=F32)


def exceptional_cases(out: dict):
    width = 5120
    for bits in (4, 8):
        rows = []
        for row in range(7):
            col = np.arange(width)
            if row == 0:
                v = np.zeros(width, F32)
            elif row == 1:
                v = np.ones(width, F32)
            elif row == 2:
                v = ((col * 37 % 257).astype(F32) - F32(128.0)) / F32(91.0)
            elif row == 3:
                v = np.where(col == 259, F32(np.nan), F32(-0.5)).astype(F32)
            elif row == 4:
                v = np.where(col == 515, F32(np.inf), F32(-0.5)).astype(F32)
            elif row == 5:
                v = np.full(width, bf16_f32(np.uint16(0x7F7F)), F32)
            else:
                v = np.full(width, np.uint32(0x00010000).view(F32), F32)
            rows.append(v)
        x = bf16_bits(np.stack(rows))
        words, scales = [], []
        for r in range(7):
            codes, s = quantize(rotated(x[r]), bits)
            words.append(pack_words(codes, bits))
            scales.append(s)
        out[f"exc_b{bits}_x"] = x
        out[f"exc_b{bits}_words"] = np.stack(words)
        out[f"exc_b{bits}_scales"] = np.array(scales, dtype=F32)


def gemm_cases(out: dict):
    """src/quantized.rs:977-1070 (bits 4 and 8; two weight matrices; rows 1 and 17)."""
    for bits in (4, 8):
        for index in (0, 1):
            i = np.arange(256 * 256, dtype=np.int64)
            w = bf16_bits((((i * (17 + index * 4)) % 251).astype(F32) - F32(125.0)) / F32(128.0)).reshape(256, 256)
            wq = [quantize(rotated(w[r]), bits) for r in range(256)]
            for rows in (1, 17):
                j = np.arange((rows + 1) * 256, dtype=np.int64)
                xin = bf16_bits(((j * 31 % 257).astype(F32) - F32(128.0)) / F32(64.0)).reshape(rows + 1, 256)
                for start in (0, 1):
                    x = xin[start:start + rows]
                    aq = [quantize(rotated(x[r]), bits) for r in range(rows)]
                    dot = np.zeros((rows, 256), dtype=np.int64)
                    exp_ = np.zeros((rows, 256), dtype=F32)
                    for r in range(rows):
                        a, a_s = aq[r]
                        for c in range(256):
                            wc, w_s = wq[c]
                            d = int(np.dot(a.astype(np.int64), wc.astype(np.int64)))
                            dot[r, c] = d
                            exp_[r, c] = bf16_f32(bf16_bits(F32(F32(F32(d) * a_s) * w_s)))
                    key = f"gemm_b{bits}_i{index}_r{rows}_s{start}"
                    out[key + "_x"] = x
                    out[key + "_dot"] = dot.astype(np.int32)
                    out[key + "_expected"] = exp_
            out[f"gemm_b{bits}_i{index}_w"] = w


def router_inputs(tokens: int, experts: int, phase: int) -> np.ndarray:
    i = np.arange(tokens * experts, dtype=np.int64)
    if phase == 0:
        v = ((i * 37 + i // experts * 11) % 257).astype(F32) / F32(16.0) - F32(8.0)
    elif phase == 1:
        v = ((i * 53 + i // experts * 7) % 5).astype(F32) - F32(2.0)
    elif phase == 2:
        v = np.where(i % 2 == 0, F32(0.0), F32(-0.0)).astype(F32)
    else:
        v = ((i * 79 + i // experts * 17) % 263).astype(F32) * F32(16.0) - F32(2048.0)
    return v.reshape(tokens, experts).astype(F32)


def serial_route(values: np.ndarray, topk: int):
    """benches/kernels/omni_route_serial.loom; exp in float64 then rounded to f32."""
    tokens, experts = values.shape
    ids = np.zeros((tokens, topk), dtype=F32)
    probs = np.zeros((tokens, topk), dtype=F32)
    for t in range(tokens):
        chosen, vals = [], []
        for r in range(topk):
            bv, bi = F32(-3.402823466e38), 0
            for e in range(experts):
                v = values[t, e]
                if e not in chosen and v > bv:
                    bv, bi = v, e
            chosen.append(bi)
            vals.append(bv)
        mx = vals[0]
        p = [F32(np.exp(np.float64(F32(v - mx)))) for v in vals]
        s = F32(0.0)
        for q in p:
            s = F32(s + q)
        ids[t] = chosen
        probs[t] = bf16_f32(bf16_bits(np.array([F32(q / s) for q in p], dtype=F32)))
    return ids, probs


def route_cases(out: dict):
    for experts, topk in ((128, 8), (64, 8), (128, 4)):
        for phase in range(4):
            v = router_inputs(5, experts, phase)
            for bf in (0, 1):
                vin = bf16_f32(bf16_bits(v)) if bf else v
                ids, probs = serial_route(vin, topk)
                # CPU stable descending sort must agree (src/benchmarking/omni.rs:74-90).
                for t in range(vin.shape[0]):
                    order = sorted(range(experts), key=lambda e: -vin[t, e])
                    assert [int(q) for q in ids[t]] == order[:topk]
                key = f"route_e{experts}_k{topk}_p{phase}_bf{bf}"
                out[key + "_logits"] = bf16_bits(vin) if bf else vin
                out[key + "_ids"] = ids
                out[key + "_probs"] = probs


def expert_routes(tokens: int, skewed: bool, phase: int, topk: int = 8) -> np.ndarray:
    """src/benchmarking/omni.rs:307-327 / src/omni.rs:917-924."""
    r = np.zeros((tokens, 2 * topk), dtype=F32)
    for t in range(tokens):
        for k in range(topk):
            r[t, k] = ((0 if skewed else t * 13) + k * 7 + phase * 19) % 128
        r[t, topk:] = 0.125
    return r


def group_cases(out: dict):
    for tokens in (1, 17, 64, 65, 128, 255, 256):
        for phase in range(3):
            routes = expert_routes(tokens, phase == 1, phase)
            groups = np.zeros((128, tokens + 1), dtype=F32)
            for e in range(128):
                members = [t * 8 + k for t in range(tokens) for k in range(8) if routes[t, k] == e]
                groups[e, 0] = len(members)
                groups[e, 1:1 + len(members)] = members
            order = np.zeros((tokens, 8), dtype=F32)
            for t in range(tokens):
                order[t] = sorted(range(8), key=lambda k: routes[t, k])
            ntask = 1 + 2 * (-(-tokens * 8 // 16) + 127)
            tasks = np.zeros(ntask, dtype=F32)
            total = 0
            for e in range(128):
                for row in range(0, int(groups[e, 0]), 16):
                    tasks[1 + 2 * total] = e
                    tasks[2 + 2 * total] = row
                    total += 1
            tasks[0] = total
            key = f"group_t{tokens}_p{phase}"
            out[key + "_routes"] = routes
            out[key + "_groups"] = groups
            out[key + "_order"] = order
            out[key + "_tasks"] = tasks


def main():
    out: dict = {}
    packing_cases(out)
    exceptional_cases(out)
    gemm_cases(out)
    route_cases(out)
    group_cases(out)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
