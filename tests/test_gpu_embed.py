"""q3s_embed_sum through the C ABI against the numpy oracle
(oracle/embed_oracle.py), the restatement of src/talker/talker.rs:568-580.

Bar: bit-exact output and status for f32 and bf16, since the kernel performs
the same additions in the same order with the same rounding.  The codebook
shapes are the 12 Hz models': codebook 0 of 3072 ids and codebooks 1..15 of
2048 ids, hidden 1024 and 2048; hidden 1000 and an unaligned text row take
the scalar path.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes
    pytest.skip("needs a CUDA device", allow_module_level=True)

import q3s  # noqa: E402
import embed_oracle as eo  # noqa: E402

DEV = torch.device("cuda:0")
VOCABS = [3072] + [2048] * 15


def _make(rng, hidden, vocabs=VOCABS, scale=0.05):
    return [(rng.standard_normal((v, hidden)) * scale).astype(np.float32) for v in vocabs]


def _to_dev(a, bf16):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:  # bf16 bit patterns
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(DEV)
    return torch.from_numpy(a).to(DEV)


def _run(codes, tables, text, bf16):
    """(device out as f32 array or bf16 bits, status) and the oracle's."""
    host_tables = [eo.f32_to_bf16(t) for t in tables] if bf16 else tables
    host_text = None if text is None else (eo.f32_to_bf16(text) if bf16 else text)
    dt = [_to_dev(t, bf16) for t in host_tables]
    dtext = None if host_text is None else _to_dev(host_text, bf16)
    dcodes = torch.from_numpy(codes.astype(np.int32)).to(DEV)
    out, status = q3s.embed_sum(dcodes, dt, dtext)
    torch.cuda.synchronize()
    got = out.cpu()
    got = got.view(torch.int16).numpy().view(np.uint16) if bf16 else got.numpy()
    ref, rst = eo.embed_sum(codes.astype(np.uint32), host_tables, host_text, bf16=bf16)
    return got, status.cpu().numpy(), ref, rst


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("hidden", [1024, 2048, 1000])
@pytest.mark.parametrize("text_kind", ["none", "row", "per_row"])
def test_embed_sum_matches_oracle(bf16, hidden, text_kind):
    rng = np.random.default_rng(hidden + 7 * bf16 + len(text_kind))
    R = 300
    tables = _make(rng, hidden)
    codes = np.stack([rng.integers(0, v, R) for v in VOCABS], 1).astype(np.uint32)
    text = {"none": None, "row": rng.standard_normal(hidden).astype(np.float32),
            "per_row": rng.standard_normal((R, hidden)).astype(np.float32)}[text_kind]
    got, st, ref, rst = _run(codes, tables, text, bf16)
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("bf16", [False, True])
def test_invalid_codes_zero_the_row(bf16):
    rng = np.random.default_rng(11)
    R, H = 64, 1024
    tables = _make(rng, H)
    codes = np.stack([rng.integers(0, v, R) for v in VOCABS], 1).astype(np.uint32)
    codes[3, 0] = 3072          # one past codebook 0
    codes[10, 15] = 2048        # one past codebook 15
    codes[20, 7] = 0xFFFFFFFF
    codes[21, 1] = 2047         # the last valid id
    got, st, ref, rst = _run(codes, tables, None, bf16)
    assert sorted(np.flatnonzero(st).tolist()) == [3, 10, 20]
    assert (st[[3, 10, 20]] == q3s.STATUS_INVALID_CODE).all()
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(got, ref)
    assert (got[[3, 10, 20]] == 0).all()


def test_strided_text_and_single_group():
    """A text operand that is a column slice (row stride 2H) and G = 1."""
    rng = np.random.default_rng(12)
    R, H = 40, 512
    tables = _make(rng, H, vocabs=[100])
    codes = rng.integers(0, 100, (R, 1)).astype(np.uint32)
    wide = torch.from_numpy(rng.standard_normal((R, 2 * H)).astype(np.float32)).to(DEV)
    text = wide[:, H:]
    out, st = q3s.embed_sum(torch.from_numpy(codes.astype(np.int32)).to(DEV),
                            [torch.from_numpy(tables[0]).to(DEV)], text)
    ref, rst = eo.embed_sum(codes, tables, text.cpu().numpy())
    np.testing.assert_array_equal(st.cpu().numpy(), rst)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_many_rows_grid_stride():
    """More rows than the grid holds, so blocks loop over rows."""
    rng = np.random.default_rng(13)
    R, H = 5000, 256
    vocabs = [64] * 16
    tables = _make(rng, H, vocabs=vocabs)
    codes = rng.integers(0, 64, (R, 16)).astype(np.uint32)
    codes[R - 1, 5] = 64
    got, st, ref, rst = _run(codes, tables, None, True)
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(got, ref)


def test_rejects_bad_arguments():
    t = torch.zeros((4, 8), device=DEV)
    c = torch.zeros((2, 1), dtype=torch.int32, device=DEV)
    with pytest.raises(TypeError):
        q3s.embed_sum(c, [t.double()])
    with pytest.raises(ValueError):
        q3s.embed_sum(c, [t, t])
    with pytest.raises(ValueError):
        q3s.embed_sum(torch.zeros((2, 33), dtype=torch.int32, device=DEV), [t] * 33)
    # Widths, shapes and devices the C entry point cannot check itself.
    t2 = torch.zeros((4, 8), device=DEV)
    c1 = torch.zeros((2, 1), dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError):
        q3s.embed_sum(c1, [t2], torch.zeros(7, device=DEV))  # 1-D text of the wrong width
    with pytest.raises(ValueError):
        q3s.embed_sum(c1, [t2], torch.zeros((2, 9), device=DEV))  # [R, H'] text
    with pytest.raises(ValueError):
        q3s.embed_sum(c1, [t2], torch.zeros((3, 8), device=DEV))  # wrong number of rows
    with pytest.raises(ValueError):
        q3s.embed_sum(c1, [t2], torch.zeros(8))  # text on the host
    with pytest.raises(ValueError):
        q3s.embed_sum(c1, [t2.cpu()])  # table on the host
    ok_out = (torch.empty((2, 8), device=DEV), torch.empty(2, dtype=torch.uint8, device=DEV))
    q3s.embed_sum(c1, [t2], out=ok_out)
    for bad in ((torch.empty((2, 9), device=DEV), ok_out[1]),
                (torch.empty((2, 8), device=DEV, dtype=torch.bfloat16), ok_out[1]),
                (torch.empty((2, 8)), ok_out[1]),
                (ok_out[0], torch.empty(3, dtype=torch.uint8, device=DEV)),
                (ok_out[0], torch.empty(2, dtype=torch.int32, device=DEV))):
        with pytest.raises(ValueError):
            q3s.embed_sum(c1, [t2], out=bad)
