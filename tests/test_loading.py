"""Weight-load policy, tiled checkpoint layout and the CLFPACK1 cache (host logic on CPU; the
device untile and load on a GPU).  Cases follow the reference's own tests:
src/checkpoint.rs:713-815 (tiled projection policy, tile/untile round trip) and
src/packed_cache.rs:197-229 (cache hits, misses, corruption)."""
import numpy as np
import pytest
import torch

from clefq.loading import (PackedWeightCache, QuantizedProjections, tile_rows, tiled_position, tiled_projection,
                           untile_rows)


def test_tiled_projection_policy():
    layer = "model.language_model.layers.3"
    assert tiled_projection(f"{layer}.mlp.up_proj.weight", 17408, 5120)
    assert tiled_projection(f"{layer}.self_attn.k_proj.weight", 1024, 5120)
    assert tiled_projection(f"{layer}.linear_attn.in_proj_qkv.weight", 10240, 5120)
    assert tiled_projection(f"{layer}.linear_attn.out_proj.weight", 5120, 6144)
    assert tiled_projection("thinker.model.layers.7.mlp.down_proj.weight", 2048, 768)
    assert not tiled_projection(f"{layer}.linear_attn.in_proj_a.weight", 48, 5120)
    assert not tiled_projection(f"{layer}.linear_attn.conv1d.weight", 10240, 4)
    assert not tiled_projection(f"{layer}.mlp.up_proj.bias", 17408, 1)
    assert not tiled_projection(f"{layer}.input_layernorm.weight", 5120, 1)
    assert not tiled_projection("model.visual.merger.linear_fc2.weight", 5120, 4608)
    assert not tiled_projection("head.memory_projection.weight", 1024, 5120)
    assert not tiled_projection("lm_head.weight", 248320, 5120)
    assert not tiled_projection(f"{layer}.mlp.up_proj.weight", 17400, 5120)
    assert not tiled_projection(f"{layer}.mlp.up_proj.weight", 17408, 5100)


def test_tile_and_untile_round_trip():
    rows, cols = 512, 192
    dense = (np.arange(rows * cols, dtype=np.int64) * 7 % 65521).astype(np.uint16).reshape(rows, cols)
    tiled = tile_rows(dense, rows, cols)
    assert tiled.size == dense.size
    for n, k in [(0, 0), (1, 0), (0, 1), (255, 63), (256, 64), (300, 150), (511, 191)]:
        assert tiled[tiled_position(cols, n, k)] == dense[n, k], (n, k)
    # each 256 x 64 block is contiguous and equal to the dense block (tile row 1, K-step 2)
    block = tiled[5 * 256 * 64:][:256 * 64].reshape(256, 64)
    assert np.array_equal(block, dense[256:512, 128:192])
    assert np.array_equal(untile_rows(tiled, rows, cols), dense)
    with pytest.raises(ValueError):
        tile_rows(dense[:, :100], rows, 100)


def test_precision_policy():
    mlp = QuantizedProjections.for_precision("int4-mlp")
    full = QuantizedProjections.for_precision("int4")
    bf16 = QuantizedProjections.for_precision("bf16")
    layer = "model.language_model.layers.0"
    assert bf16.is_bf16() and not mlp.is_bf16() and full.is_full_int4() and not mlp.is_full_int4()
    for proj in ("gate", "up", "down"):
        assert mlp.precision(f"{layer}.mlp.{proj}_proj.weight", 17408, 5120) == 4
        assert full.precision(f"{layer}.mlp.{proj}_proj.weight", 17408, 5120) == 4
    assert mlp.precision(f"{layer}.self_attn.q_proj.weight", 6144, 5120) is None
    assert full.precision(f"{layer}.self_attn.q_proj.weight", 6144, 5120) == 4
    assert full.precision(f"{layer}.self_attn.k_proj.weight", 1024, 5120) is None   # rows < 4096
    assert full.precision(f"{layer}.linear_attn.conv1d.weight", 10240, 4) is None
    assert full.precision("lm_head.weight", 248320, 5120) is None
    assert full.precision(f"{layer}.mlp.up_proj.bias", 17408, 256) is None
    assert bf16.precision(f"{layer}.mlp.up_proj.weight", 17408, 5120) is None
    only_up = QuantizedProjections(bits=8, projections=("up",))
    assert only_up.precision(f"{layer}.mlp.up_proj.weight", 512, 512) == 8
    assert only_up.precision(f"{layer}.mlp.down_proj.weight", 512, 512) is None
    assert full.resident_bytes(f"{layer}.mlp.up_proj.weight", 17408, 5120) == 17408 * 5120 // 2 + 17408 * 4
    assert mlp.resident_bytes(f"{layer}.self_attn.q_proj.weight", 6144, 5120) == 6144 * 5120 * 2


def test_packed_cache_hits_misses_and_corruption(tmp_path):
    cache = PackedWeightCache(tmp_path, "compiler-a", "sm_100a")
    key = cache.key("weight", 256, 256, 4, b"source")
    assert cache.read(key) is None
    codes, scales = bytes([0x5A]) * 32768, bytes([0x17]) * 1024
    cache.write(key, codes, scales)
    assert cache.read(key) == (codes, scales)
    assert (cache.hits, cache.misses) == (1, 1)
    assert cache.read(cache.key("weight", 256, 256, 4, b"changed source")) is None
    other = PackedWeightCache(tmp_path, "compiler-b", "sm_100a")
    assert other.read(other.key("weight", 256, 256, 4, b"source")) is None
    raw = cache.path(key).read_bytes()
    assert raw[:8] == b"CLFPACK1" and int.from_bytes(raw[8:12], "little") + 12 + 32768 + 1024 == len(raw)
    bad = bytearray(raw)
    bad[-1] ^= 1
    cache.path(key).write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="checksum"):
        cache.read(key)
    cache.path(key).write_bytes(bytes(bad[:-1]))
    with pytest.raises(ValueError, match="length"):
        cache.read(key)
    with pytest.raises(ValueError):
        cache.write(key, codes[:-1], scales)


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols,bits", [(256, 512, 4), (768, 1024, 4), (512, 2048, 8)])
def test_device_untile_and_tiled_load(rows, cols, bits):
    import clefq
    from oracle import oracle as o
    rng = np.random.default_rng(rows + cols)
    dense = o.f32_to_bf16((rng.standard_normal((rows, cols)) * 0.05).astype(np.float32))
    tiled = tile_rows(dense, rows, cols)
    dev_tiled = torch.from_numpy(tiled.view(np.int16).copy()).view(torch.bfloat16).cuda().view(rows, cols)
    back = clefq.untile_bf16(dev_tiled)
    assert np.array_equal(back.view(torch.int16).cpu().numpy().view(np.uint16), dense)
    dev_dense = torch.from_numpy(dense.view(np.int16).copy()).view(torch.bfloat16).cuda()
    a = clefq.load_quantized_weight(dev_dense, bits)
    b = clefq.load_quantized_weight(dev_tiled, bits, tiled=True)
    assert torch.equal(a.codes, b.codes) and torch.equal(a.scales.view(torch.int32), b.scales.view(torch.int32))
    ref_codes, ref_scales = o.pack_weight(dense, bits)
    assert np.array_equal(a.codes.cpu().numpy().view(np.uint32).ravel(), np.asarray(ref_codes).ravel())
    assert np.array_equal(a.scales.cpu().numpy().view(np.uint32), np.asarray(ref_scales, np.float32).view(np.uint32))
