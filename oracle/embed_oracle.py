"""ORACLE — test infrastructure only.  numpy restatement of the codebook
embedding sum that follows sampling in the reference (qwen3tts-rs 0.2.0,
src/talker/talker.rs:568-580; embedding_lookup: src/talker/primitives.rs:17-25):

    sum = T0[c0]; for g in 1..G: sum = sum + Tg[cg]; next = sum + text

Each addition is one tensor add in the model dtype (candle binary add,
patches/candle-kernels/src/binary.cu:5), so every partial sum is rounded to
that dtype: f32 adds for f32; for bf16, the f32 sum of the two bf16 values
rounded to bf16 (round to nearest even), which is the correctly rounded bf16
sum.  A code at or beyond its codebook's vocabulary makes the reference's
index_select fail; here that row gets status 8 and zeros.

bf16 values are carried as uint16 bit patterns.
"""
from __future__ import annotations

import numpy as np

STATUS_OK = 0
STATUS_INVALID_CODE = 8


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round f32 to bf16 bits, nearest even (NaN -> quiet NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r)


def embed_sum(codes: np.ndarray, tables, text=None, bf16: bool = False):
    """codes [R, G] (uint32); tables: G arrays [V_g, H] (float32, or uint16
    bf16 bits when bf16); text None, [H] or [R, H] of the same kind.
    Returns (out [R, H] float32 or uint16 bits, status [R] uint8)."""
    codes = np.asarray(codes, dtype=np.uint64)
    R, G = codes.shape
    H = tables[0].shape[1]
    status = np.zeros(R, np.uint8)
    bad = np.zeros(R, bool)
    for g in range(G):
        bad |= codes[:, g] >= tables[g].shape[0]
    status[bad] = STATUS_INVALID_CODE
    safe = np.where(bad[:, None], 0, codes).astype(np.int64)

    def val(a):
        return bf16_to_f32(a) if bf16 else a.astype(np.float32)

    def rnd(x):
        return bf16_to_f32(f32_to_bf16(x)) if bf16 else x

    acc = val(tables[0][safe[:, 0]])
    for g in range(1, G):
        acc = rnd((acc + val(tables[g][safe[:, g]])).astype(np.float32))
    if text is not None:
        t = val(np.asarray(text))
        acc = rnd((acc + (t if t.ndim == 2 else t[None, :])).astype(np.float32))
    acc[bad] = 0.0
    out = f32_to_bf16(acc) if bf16 else acc.astype(np.float32)
    return out, status
