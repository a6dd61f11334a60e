"""Readers for the golden vectors in tests/golden/ (written by make_golden.py)."""
import json
import struct
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


def bits_to_f32(bits: str) -> float:
    return struct.unpack("<f", struct.pack("<I", int(bits, 16) & 0xFFFFFFFF))[0]


def f32_bits(x) -> str:
    return "0x%08x" % struct.unpack("<I", struct.pack("<f", float(x)))[0]


def decode_row(row: dict) -> np.ndarray:
    """Inverse of make_golden.encode_row."""
    out = np.full(row["n"], np.uint32(int(row["fill"], 16)), dtype=np.uint32)
    for i, b in row["at"]:
        out[i] = np.uint32(int(b, 16))
    return out.view(np.float32)


def decode_q64(values) -> np.ndarray:
    out = []
    for v in values:
        if v == "nan":
            out.append(float("nan"))
        elif v == "-inf":
            out.append(float("-inf"))
        else:
            out.append(v / 64.0)
    return np.array(out, dtype=np.float32)
