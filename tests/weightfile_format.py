"""Test infrastructure: GoTransformers binary weights files written the way
the reference writes them (weightfile/binaryfile.go), to feed the library's
loader (gtmoe_weightfile_*).

Format (binaryfile.go:13-21, 63-138): a 24-byte marker
("GOTRANSFORMERS-WEIGHTS-1" or "-2"), a uint32 parameter count, then per
parameter a uint32 name length and the name; version 1 stores a uint64 count
and float64 values; version 2 a storage byte (1 float64, 2 float32,
3 bfloat16, 4 compressed rows) and then the values, or for compressed rows
(writeCompressedRows, :127-138) the precision byte, uint64 rows, uint64
width and five count-prefixed lists (float64, float32, int8, fp4 bytes,
float32 scales).  All little-endian."""
from __future__ import annotations

import math
import struct

import numpy as np

MARKER_V1 = b"GOTRANSFORMERS-WEIGHTS-1"
MARKER_V2 = b"GOTRANSFORMERS-WEIGHTS-2"
FLOAT64, FLOAT32, BFLOAT16, COMPRESSED = 1, 2, 3, 4


def bf16_bits(value: float) -> int:
    """float64ToBFloat16Bits (weightfile/precision.go:58-71): round to the
    nearest bfloat16, ties to even, with bfloat16's own subnormal spacing."""
    if math.isnan(value):
        return 0x7FC0
    if value == 0 or math.isinf(value):
        return struct.unpack("<I", struct.pack("<f", value))[0] >> 16
    _, e = math.frexp(value)
    exponent = max(e - 1, -126)
    spacing = exponent - 7
    steps = round(math.ldexp(value, -spacing))  # Python rounds halves to even, as math.RoundToEven
    rounded = math.ldexp(steps, spacing)
    return struct.unpack("<I", struct.pack("<f", rounded))[0] >> 16


def _count_and_values(out: bytearray, values: np.ndarray, dtype) -> None:
    arr = np.ascontiguousarray(values, dtype=dtype).reshape(-1)
    out += struct.pack("<Q", arr.size)
    out += arr.astype(np.dtype(dtype).newbyteorder("<")).tobytes()


def compressed_record(precision: int, rows: int, width: int, values: np.ndarray, scales=None) -> tuple:
    """A lowprecision.RowsSnapshot: only the list of `precision` (and the
    scales for Int8/FP4) is non-empty."""
    return ("rows", precision, rows, width, values, scales)


def write(path: str, params: list, version: int = 2) -> None:
    """params: [(name, entry)], entry = ("f64"|"f32"|"bf16", values) or a
    compressed_record(...)."""
    out = bytearray(MARKER_V1 if version == 1 else MARKER_V2)
    out += struct.pack("<I", len(params))
    for name, entry in params:
        nb = name.encode()
        out += struct.pack("<I", len(nb)) + nb
        kind = entry[0]
        if version == 1:
            _count_and_values(out, entry[1], np.float64)
            continue
        if kind == "f64":
            out += bytes([FLOAT64])
            _count_and_values(out, entry[1], np.float64)
        elif kind == "f32":
            out += bytes([FLOAT32])
            _count_and_values(out, np.asarray(entry[1], np.float64).astype(np.float32), np.float32)
        elif kind == "bf16":
            out += bytes([BFLOAT16])
            bits = np.array([bf16_bits(float(v)) for v in np.asarray(entry[1]).reshape(-1)], np.uint16)
            _count_and_values(out, bits, np.uint16)
        else:
            _, precision, rows, width, values, scales = entry
            out += bytes([COMPRESSED, precision]) + struct.pack("<QQ", rows, width)
            empty = np.zeros(0)
            lists = {0: np.float64, 1: np.float32, 2: np.int8, 3: np.uint8}
            for p, dt in lists.items():
                _count_and_values(out, values if p == precision else empty, dt)
            _count_and_values(out, scales if scales is not None else empty, np.float32)
    with open(path, "wb") as f:
        f.write(out)
