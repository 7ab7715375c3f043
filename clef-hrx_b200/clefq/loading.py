"""Weight-load policy and on-disk formats of the INT4 path.

- `QuantizedProjections`: which checkpoint tensors become packed integer weights and at what
  width (src/quantized.rs:22-127: `precision`, `resident_bytes`, `for_precision`).
- `tiled_projection`, `tile_rows`, `untile_rows`: the checkpoint's tiled256x64 layout of the
  text-backbone projections (src/checkpoint.rs:20-100); the device path restores rows with
  `clefq.untile_bf16` / `clefq.load_quantized_weight(..., tiled=True)`.
- `load_weight`: the policy plus the device load in one call (src/quantized.rs:147-234).
- `PackedWeightCache`: the CLFPACK1 cache of packed weight bytes (src/packed_cache.rs:13-230):
  `CLFPACK1`, u32 LE header length, a JSON header (the key plus SHA-256 of codes and scales),
  the tiled codes, the f32 scales; one file per key, named by the SHA-256 of the key's JSON.
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

TILED_LAYOUT = "tiled256x64"
TILE_ROWS, TILE_COLS = 256, 64
_PROJECTIONS = ("q_proj", "k_proj", "v_proj", "o_proj", "in_proj_qkv", "in_proj_z", "out_proj", "gate_proj",
                "up_proj", "down_proj")


# ---------------------------------------------------------------------------------------
# precision policy (src/quantized.rs:22-127)
# ---------------------------------------------------------------------------------------
@dataclass
class QuantizedProjections:
    """bits: width of the selected MLP projections (INT4-MLP mode); backbone_bits: width of
    every large backbone matrix (INT4 mode); projections: the MLP projections covered."""
    bits: int | None = None
    backbone_bits: int | None = None
    projections: tuple = ("up", "gate", "down")

    @classmethod
    def for_precision(cls, precision: str) -> "QuantizedProjections":
        """precision: "bf16", "int4-mlp" or "int4" (src/quantized.rs:54-61)."""
        if precision not in ("bf16", "int4-mlp", "int4"):
            raise ValueError(f"unknown precision {precision!r}")
        return cls(bits=4 if precision == "int4-mlp" else None, backbone_bits=4 if precision == "int4" else None)

    def is_bf16(self) -> bool:
        return self.bits is None and self.backbone_bits is None

    def is_full_int4(self) -> bool:
        return self.bits is None and self.backbone_bits == 4 and tuple(self.projections) == ("up", "gate", "down")

    def precision(self, name: str, rows: int, cols: int) -> int | None:
        """Bits of the packed weight for this tensor, or None to keep it BF16."""
        if not name.startswith("model.language_model.layers.") or not name.endswith(".weight"):
            return None
        if ".mlp." in name:
            if any(name.endswith(f".{p}_proj.weight") for p in self.projections):
                return self.bits if self.bits is not None else self.backbone_bits
            return None
        if rows >= 4096 and cols >= 1024 and rows % 256 == 0 and cols % 256 == 0:
            return self.backbone_bits
        return None

    def resident_bytes(self, name: str, rows: int, cols: int) -> int:
        """Device bytes of the tensor once loaded: tiled codes (no stride padding) plus one f32
        scale per row, or BF16."""
        bits = self.precision(name, rows, cols)
        return rows * cols * bits // 8 + rows * 4 if bits is not None else rows * cols * 2


# ---------------------------------------------------------------------------------------
# tiled checkpoint layout (src/checkpoint.rs:20-100)
# ---------------------------------------------------------------------------------------
def tiled_projection(name: str, rows: int, cols: int) -> bool:
    """Whether the checkpoint stores this tensor in the tiled256x64 layout."""
    if rows <= 0 or cols <= 0 or rows % TILE_ROWS or cols % TILE_COLS:
        return False
    for prefix in ("model.language_model.layers.", "thinker.model.layers."):
        if name.startswith(prefix):
            rest = name[len(prefix):]
            break
    else:
        return False
    if not rest.endswith(".weight"):
        return False
    return rest[: -len(".weight")].rsplit(".", 1)[-1] in _PROJECTIONS


def tiled_position(cols: int, n: int, k: int) -> int:
    """Element index of logical (n, k) in the tiled layout."""
    return (((n // TILE_ROWS) * (cols // TILE_COLS) + k // TILE_COLS) * TILE_ROWS + n % TILE_ROWS) * TILE_COLS + \
        k % TILE_COLS


def _check_tiled(a: np.ndarray, rows: int, cols: int) -> np.ndarray:
    if rows % TILE_ROWS or cols % TILE_COLS:
        raise ValueError("tiled layout requires 256-row and 64-column multiples")
    a = np.ascontiguousarray(a).reshape(-1)
    if a.size != rows * cols:
        raise ValueError("BF16 element count")
    return a


def tile_rows(a: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Row-major [rows][cols] 16-bit elements -> tiled order (flat)."""
    a = _check_tiled(a, rows, cols)
    t = a.reshape(rows // TILE_ROWS, TILE_ROWS, cols // TILE_COLS, TILE_COLS)
    return np.ascontiguousarray(t.transpose(0, 2, 1, 3)).reshape(-1)


def untile_rows(a: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Tiled order (flat) -> row-major [rows][cols]."""
    a = _check_tiled(a, rows, cols)
    t = a.reshape(rows // TILE_ROWS, cols // TILE_COLS, TILE_ROWS, TILE_COLS)
    return np.ascontiguousarray(t.transpose(0, 2, 1, 3)).reshape(rows, cols)


def load_weight(policy: QuantizedProjections, name: str, w, tiled: bool | None = None):
    """Packs one checkpoint tensor (a CUDA BF16 tensor of logical shape [rows][cols], in the
    checkpoint's byte order) when the policy selects it: returns a `clefq.QuantizedWeight`, or
    None for a tensor that stays BF16 (src/quantized.rs:147-160)."""
    from . import load_quantized_weight
    rows, cols = w.shape
    bits = policy.precision(name, rows, cols)
    if bits is None:
        return None
    if rows % 256 or cols % 256:
        raise ValueError("unsupported quantized weight shape")
    if tiled is None:
        tiled = tiled_projection(name, rows, cols)
    return load_quantized_weight(w, bits, tiled=tiled)


# ---------------------------------------------------------------------------------------
# CLFPACK1 packed-weight cache (src/packed_cache.rs:13-230)
# ---------------------------------------------------------------------------------------
MAGIC = b"CLFPACK1"
_MAX_HEADER = 65536


def _digest(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def _json(obj) -> bytes:
    """Compact JSON with fields in declaration order (the key's identity is its bytes)."""
    return json.dumps(obj, separators=(",", ":"), ensure_ascii=False).encode()


def packing_identity() -> str:
    """Identity of this build's packing: its layout tag and the sources that define the bytes
    (a change of either misses every cached entry).  It hashes this build's own sources, so
    cache files written by the reference (whose identity hashes its kernels) never match
    here, and the reverse: the file format is shared, the entries are not."""
    here = Path(__file__).resolve().parent.parent / "csrc"
    h = hashlib.sha256(b"tiled256x64-to-rotated-codes128x32-v1\n")
    for name in ("prepare.cu", "cq_math.h", "cq_common.cuh", "load.cu"):
        f = here / name
        if f.exists():
            h.update(f.read_bytes())
    return h.hexdigest()


@dataclass
class CacheKey:
    name: str
    rows: int
    cols: int
    bits: int
    compiler: str
    target: str
    source_sha256: str
    packing_sha256: str

    def as_dict(self) -> dict:
        return {"name": self.name, "rows": self.rows, "cols": self.cols, "bits": self.bits,
                "compiler": self.compiler, "target": self.target, "source_sha256": self.source_sha256,
                "packing_sha256": self.packing_sha256}

    def sizes(self) -> tuple[int, int]:
        if self.bits not in (4, 8) or self.rows <= 0 or self.cols <= 0 or self.rows % 256 or self.cols % 256:
            raise ValueError("invalid packed-cache extent")
        return self.rows * self.cols * self.bits // 8, self.rows * 4


class PackedWeightCache:
    def __init__(self, directory, compiler: str, target: str, packing: str | None = None):
        self.directory = Path(directory)
        self.compiler = compiler
        self.target = target
        self.packing = packing if packing is not None else packing_identity()
        self.hits = 0
        self.misses = 0

    def key(self, name: str, rows: int, cols: int, bits: int, source: bytes) -> CacheKey:
        return CacheKey(name, rows, cols, bits, self.compiler, self.target, _digest(source), self.packing)

    def path(self, key: CacheKey) -> Path:
        return self.directory / f"{_digest(_json(key.as_dict()))}.pack"

    def read(self, key: CacheKey):
        """(codes bytes, scales bytes), or None on a miss; a damaged file raises."""
        path = self.path(key)
        try:
            f = open(path, "rb")
        except FileNotFoundError:
            self.misses += 1
            return None
        with f:
            code_bytes, scale_bytes = key.sizes()
            prefix = f.read(12)
            if len(prefix) < 12:
                raise ValueError("truncated packed-cache prefix")
            if prefix[:8] != MAGIC:
                raise ValueError("invalid packed-cache magic")
            header_bytes = int.from_bytes(prefix[8:], "little")
            if header_bytes > _MAX_HEADER:
                raise ValueError("oversized packed-cache header")
            if os.fstat(f.fileno()).st_size != 12 + header_bytes + code_bytes + scale_bytes:
                raise ValueError("packed-cache length mismatch")
            header = json.loads(f.read(header_bytes))
            if header.get("key") != key.as_dict():
                raise ValueError("packed-cache key mismatch")
            codes = f.read(code_bytes)
            scales = f.read(scale_bytes)
        if _digest(codes) != header.get("codes_sha256") or _digest(scales) != header.get("scales_sha256"):
            raise ValueError(f"packed-cache checksum mismatch: {path}")
        self.hits += 1
        return codes, scales

    def write(self, key: CacheKey, codes: bytes, scales: bytes):
        if key.sizes() != (len(codes), len(scales)):
            raise ValueError("packed-cache data size mismatch")
        header = _json({"key": key.as_dict(), "codes_sha256": _digest(codes), "scales_sha256": _digest(scales)})
        if len(header) > _MAX_HEADER:
            raise ValueError("oversized packed-cache header")
        self.directory.mkdir(parents=True, exist_ok=True)
        path = self.path(key)
        temporary = path.with_suffix(f".tmp.{os.getpid()}.{id(codes)}")
        try:
            with open(temporary, "xb") as f:
                f.write(MAGIC)
                f.write(len(header).to_bytes(4, "little"))
                f.write(header)
                f.write(codes)
                f.write(scales)
                f.flush()
                os.fsync(f.fileno())
            os.replace(temporary, path)
        except BaseException:
            try:
                os.remove(temporary)
            except OSError:
                pass
            raise
