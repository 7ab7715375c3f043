"""Helpers shared by the GPU parity tests: numpy <-> torch BF16 bit patterns, seeded inputs."""
import numpy as np
import torch


def to_dev_bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).cuda()


def from_dev_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bf16_normal(rng, shape, scale=1.0):
    from oracle import oracle as o
    return o.f32_to_bf16((rng.standard_normal(shape) * scale).astype(np.float32))


def same_bits_f32(a, b) -> bool:
    a = np.asarray(a, dtype=np.float32).view(np.uint32)
    b = np.asarray(b, dtype=np.float32).view(np.uint32)
    return np.array_equal(a, b)


def permuted_operand(codes_words: np.ndarray, width: int) -> np.ndarray:
    """The s8 GEMM operand the prepare kernel writes for packed int4 rows: 16*code, within
    each 32-code group the low nibbles of its four words first, then the high nibbles."""
    w = np.ascontiguousarray(codes_words[:, : width // 8]).astype(np.uint32)
    lo = ((w << 4) & 0xF0F0F0F0).astype(np.uint32)
    hi = (w & 0xF0F0F0F0).astype(np.uint32)
    rows = w.shape[0]
    lo = lo.reshape(rows, -1, 4)
    hi = hi.reshape(rows, -1, 4)
    return np.concatenate([lo, hi], axis=2).reshape(rows, -1).view(np.int8).reshape(rows, width)


def bf16_equal_nan(a, b) -> bool:
    """Bit equality of BF16 arrays where any two NaNs count as equal (NaN payloads are not
    part of the contract: the GPU produces canonical NaNs, the host propagates payloads)."""
    from oracle import oracle as o
    a = np.asarray(a, dtype=np.uint16)
    b = np.asarray(b, dtype=np.uint16)
    na, nb = np.isnan(o.bf16_to_f32(a)), np.isnan(o.bf16_to_f32(b))
    return np.array_equal(na, nb) and np.array_equal(a[~na], b[~nb])
