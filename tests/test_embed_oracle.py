"""The codebook embedding-sum oracle (oracle/embed_oracle.py) on CPU.

The reference adds one codebook embedding at a time in the model dtype
(src/talker/talker.rs:568-580), each add a candle binary add that rounds its
result to the dtype.  torch's CPU add of two bf16 tensors does the same (f32
add, round to nearest even), so it pins the oracle's bf16 arithmetic; for f32
the sum order is the only thing to pin.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import embed_oracle as eo  # noqa: E402


def _tables(rng, groups, vocab, hidden, scale=0.05):
    return [(rng.standard_normal((vocab, hidden)) * scale).astype(np.float32)
            for _ in range(groups)]


def _torch_sum(codes, tables, text, dtype):
    acc = torch.from_numpy(tables[0][codes[:, 0]]).to(dtype)
    for g in range(1, len(tables)):
        acc = acc + torch.from_numpy(tables[g][codes[:, g]]).to(dtype)
    if text is not None:
        t = torch.from_numpy(text).to(dtype)
        acc = acc + (t if t.dim() == 2 else t[None, :])
    return acc


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 100000),
                        np.array([0.0, -0.0, np.inf, -np.inf, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8,
                                  3.3895314e38, 1e-40], np.float32)]).astype(np.float32)
    got = eo.f32_to_bf16(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(got, ref)
    nan = eo.f32_to_bf16(np.array([np.nan], np.float32))
    assert np.isnan(eo.bf16_to_f32(nan))[0]


@pytest.mark.parametrize("text_kind", ["none", "row", "per_row"])
def test_bf16_sum_matches_torch_sequential_adds(text_kind):
    rng = np.random.default_rng(2)
    G, V, H, R = 16, 2048, 64, 40
    tables = _tables(rng, G, V, H)
    codes = rng.integers(0, V, (R, G)).astype(np.uint32)
    text = None
    if text_kind == "row":
        text = rng.standard_normal(H).astype(np.float32)
    elif text_kind == "per_row":
        text = rng.standard_normal((R, H)).astype(np.float32)
    bits = [eo.f32_to_bf16(t) for t in tables]
    tbits = None if text is None else eo.f32_to_bf16(text)
    out, status = eo.embed_sum(codes, bits, tbits, bf16=True)
    assert (status == eo.STATUS_OK).all()
    # torch sees the tables already rounded to bf16, as the device does.
    rt = [eo.bf16_to_f32(b) for b in bits]
    rtext = None if tbits is None else eo.bf16_to_f32(tbits)
    ref = _torch_sum(codes, rt, rtext, torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(out, ref)
    # The order matters: a pairwise sum differs on some elements.
    pair = torch.stack([torch.from_numpy(t[codes[:, g]]).to(torch.bfloat16)
                        for g, t in enumerate(rt)]).float().sum(0).to(torch.bfloat16)
    if text is None:
        assert (pair.view(torch.int16).numpy().view(np.uint16) != out).any()


def test_f32_sum_order_and_invalid_codes():
    rng = np.random.default_rng(3)
    G, V, H, R = 4, 100, 8, 6
    tables = _tables(rng, G, V, H, scale=1.0)
    codes = rng.integers(0, V, (R, G)).astype(np.uint32)
    codes[2, 3] = V          # one past the codebook
    codes[4, 0] = 0xFFFFFFFF
    text = rng.standard_normal((R, H)).astype(np.float32)
    out, status = eo.embed_sum(codes, tables, text)
    assert status.tolist() == [0, 0, 8, 0, 8, 0]
    assert (out[[2, 4]] == 0).all()
    for r in (0, 1, 3, 5):
        acc = tables[0][codes[r, 0]].copy()
        for g in range(1, G):
            acc = (acc + tables[g][codes[r, g]]).astype(np.float32)
        acc = (acc + text[r]).astype(np.float32)
        np.testing.assert_array_equal(out[r], acc)


def test_codebooks_of_different_sizes():
    rng = np.random.default_rng(4)
    tables = [rng.standard_normal((v, 4)).astype(np.float32) for v in (10, 3, 7)]
    codes = np.array([[9, 2, 6], [9, 3, 6], [0, 0, 7]], np.uint32)
    out, status = eo.embed_sum(codes, tables)
    assert status.tolist() == [0, 8, 8]
    np.testing.assert_array_equal(out[0], (tables[0][9] + tables[1][2]) + tables[2][6])
