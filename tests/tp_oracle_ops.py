"""CPU stand-ins for the device steps of the tensor-parallel MLP (test infrastructure only).
GEMMs and SwiGLU come from the oracle; the split packing (shard row maxima, quantisation with
a given maximum) is written here in numpy float32 from the reference's algorithm
(kernels/prepare_integer.loom:55-291: radix-4 Hadamard in stride order 1, 4, 16, 64, then
scale = max(m * 0.0625, 1e-30) / 7, codes = rint(h * (0.0625 / scale)))."""
import numpy as np
import torch

from oracle import oracle as o


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16_tensor(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def hadamard256(v: np.ndarray) -> np.ndarray:
    """Rows of f32 values, each 256-group rotated with the reference's rounding order."""
    m, w = v.shape
    g = v.reshape(m, w // 256, 256).astype(np.float32).copy()
    for s in (1, 4, 16, 64):
        q = g.reshape(m, w // 256, 256 // (4 * s), 4, s)
        a, b, c, d = q[:, :, :, 0, :], q[:, :, :, 1, :], q[:, :, :, 2, :], q[:, :, :, 3, :]
        s01, s23, d01, d23 = a + b, c + d, a - b, c - d
        g = np.stack([s01 + d23, s01 - d23, d01 + s23, s23 - d01], axis=3).reshape(m, w // 256, 256)
    return g.reshape(m, w)


def _hidden(gu: torch.Tensor) -> np.ndarray:
    h = _u16(gu)
    n = h.shape[1] // 2
    return hadamard256(o.bf16_to_f32(o.swiglu(h[:, :n], h[:, n:])))


class OracleTpOps:
    def pack_x(self, x):
        _, codes, scales, _ = o.prepare(_u16(x), 4, o.stride_for(x.shape[1]))
        return codes.copy(), scales.copy()

    def gate_up(self, xq, m, shard):
        codes, scales = xq
        n = shard.inter // shard.world
        g = o.gemm(codes, scales, shard.gate[0], shard.gate[1], n, shard.hidden)
        u = o.gemm(codes, scales, shard.up[0], shard.up[1], n, shard.hidden)
        return _bf16_tensor(np.concatenate([g, u], axis=1))

    def rowmax(self, gu):
        a = np.abs(_hidden(gu))
        a = np.where(np.isfinite(a), a, np.float32(np.inf))
        return torch.from_numpy(a.max(axis=1).astype(np.float32))

    def pack_hidden(self, gu, rowmax):
        v = _hidden(gu)
        mx = rowmax.numpy().astype(np.float32)
        scale = (np.maximum(mx * np.float32(0.0625), np.float32(1e-30)) / np.float32(7)).astype(np.float32)
        valid = scale < np.float32(np.inf)
        inv = (np.float32(0.0625) / np.where(valid, scale, np.float32(1))).astype(np.float32)
        c = np.rint((v * inv[:, None]).astype(np.float32))
        c = np.where(valid[:, None], np.clip(c, -7, 7), 0).astype(np.int64)
        nib = (c & 0xF).astype(np.uint32).reshape(v.shape[0], -1, 8)
        words = np.zeros(nib.shape[:2], dtype=np.uint32)
        for i in range(8):
            words |= nib[:, :, i] << np.uint32(4 * i)
        return torch.from_numpy(words.view(np.int32)), torch.from_numpy(scale)

    def gather_unpack(self, codes_all, inter):
        return torch.cat(list(codes_all.unbind(0)), dim=1)   # full int4 code rows for the oracle GEMM

    def down(self, codes, scales, shard, residual):
        hs = shard.hidden // shard.world
        res = None
        if residual is not None:
            res = _u16(residual)[:, shard.rank * hs:(shard.rank + 1) * hs].copy()
        out = o.gemm(codes.numpy().view(np.uint32), scales.numpy(), shard.down[0], shard.down[1], hs, shard.inter,
                     residual=res)
        return _bf16_tensor(out)

    def interleave(self, out_all):
        return torch.cat(list(out_all.unbind(0)), dim=1)
