"""CPU stand-ins for the device steps of the expert-parallel MoE layer, built on the oracle
(test infrastructure only).  They let `clefq.ep.omni_moe_ep` run its real host logic
(count exchange, split sizes, record and product exchange, slot bookkeeping) on gloo ranks
without a GPU."""
import numpy as np
import torch

from oracle import oracle as o


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def record_bytes(hidden: int) -> int:
    return ((hidden // 8 + 3) * 4 + 15) // 16 * 16


class OracleEpOps:
    def route(self, logits, topk):
        return torch.from_numpy(o.route(_u16(logits), topk))

    def pack_tokens(self, x):
        _, codes, scales, _ = o.prepare(_u16(x), 4, o.stride_for(x.shape[1]))
        return torch.from_numpy(codes.view(np.int32).copy()), torch.from_numpy(scales.copy())

    def plan(self, routes, topk, experts, world):
        e = routes[:, :topk].numpy().astype(np.int64).ravel()
        dest = e // (experts // world)
        slots = np.zeros(e.size, dtype=np.int32)
        counts = np.zeros(world, dtype=np.int64)
        base = 0
        for d in range(world):
            idx = np.nonzero(dest == d)[0]
            slots[idx] = base + np.arange(idx.size)
            counts[d] = idx.size
            base += idx.size
        return torch.from_numpy(counts), torch.from_numpy(slots)

    def record_bytes(self, hidden):
        return record_bytes(hidden)

    def pack_records(self, codes, scales, routes, topk, slots, n_send, hidden):
        hw = hidden // 8
        rw = record_bytes(hidden) // 4
        c = codes.numpy().view(np.uint32)
        r = routes.numpy()
        recs = np.zeros((max(n_send, 1), rw), dtype=np.uint32)
        for i, slot in enumerate(slots.numpy()[: r.shape[0] * topk]):
            t, k = divmod(i, topk)
            recs[slot, :hw] = c[t, :hw]
            recs[slot, hw] = np.float32(scales[t]).view(np.uint32)
            recs[slot, hw + 1] = np.uint32(int(r[t, k]))
            recs[slot, hw + 2] = np.float32(r[t, topk + k]).view(np.uint32)
        return torch.from_numpy(recs.view(np.uint8).ravel().copy())

    def experts(self, records, n, hidden, shard):
        hw = hidden // 8
        rw = record_bytes(hidden) // 4
        out = np.zeros((max(n, 1), hidden), dtype=np.uint16)
        if n:
            recs = records.numpy().view(np.uint32).reshape(-1, rw)[:n]
            codes = recs[:, :hw].copy()
            scales = recs[:, hw].view(np.float32).copy()
            probs = recs[:, hw + 2].view(np.float32).copy()
            routes = np.stack([(recs[:, hw + 1].astype(np.int64) - shard.base).astype(np.float32), probs], axis=1)
            groups, _ = o.group(routes, shard.count)
            inter = shard.inter
            g = o.expert(codes, scales, shard.gate[0], shard.gate[1], groups, n, hidden, inter, False, 1, shard.count)
            u = o.expert(codes, scales, shard.up[0], shard.up[1], groups, n, hidden, inter, False, 1, shard.count)
            hid = o.swiglu(g, u)
            _, hc, hs, _ = o.prepare(hid, 4, o.stride_for(inter))
            vals = o.expert(hc, hs, shard.down[0], shard.down[1], groups, n, inter, hidden, True, 1, shard.count)
            out[:n] = o.f32_to_bf16(o.bf16_to_f32(vals) * probs[:, None])
        return torch.from_numpy(out.view(np.int16)).view(torch.bfloat16)

    def combine(self, products, slots, routes, topk, hidden):
        tokens = routes.shape[0]
        prod = _u16(products)
        vals = prod[slots.numpy()[: tokens * topk]]
        unit = routes.numpy().copy()
        unit[:, topk:] = 1.0
        out = o.combine(vals, unit)
        return torch.from_numpy(out.view(np.int16)).view(torch.bfloat16)
