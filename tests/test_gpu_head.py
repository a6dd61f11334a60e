"""Producer fusion (q3s_head_sample): the head projection of the talker's
codec_head / a code-predictor lm_head (logits = hidden · weightᵀ,
primitives.rs:32-42) and the sampling of its rows in one launch.

Bar: the logits within the f32 summation bound of a float64 product of the
same bf16 weights and hidden values (the reference's own matmul rounds in an
order of its library's choosing, so no bit pattern is canonical); the ids,
statuses and counters bit-exact against q3s_sample_batch and the oracle on
the returned logits.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes
    pytest.skip("needs a CUDA device", allow_module_level=True)

import q3s  # noqa: E402
import oracle  # noqa: E402

DEV = torch.device("cuda:0")


def _inputs(R, V, H, hdt, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    weight = (torch.randn((V, H), generator=g, device=DEV) * 0.05).to(torch.bfloat16)
    hidden = torch.randn((R, H), generator=g, device=DEV).to(hdt)
    return hidden, weight


def _rows(R, V, seed, talker=True):
    rng = np.random.default_rng(seed)
    if talker:
        p = q3s.make_params(R, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.05,
                            suppress_from=2048, allow_token=2150)
        if R > 2:
            p["top_k"][1] = 0
            p["top_p"][1] = 0.8           # nucleus row
            p["do_sample"][2] = 0         # greedy row
    else:
        p = q3s.make_params(R, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.0)
    lens = rng.integers(0, 300, R) if talker else np.zeros(R, np.int64)
    hoff = np.zeros(R + 1, np.int64)
    hoff[1:] = np.cumsum(lens)
    hist = rng.integers(0, 2048, int(hoff[-1])).astype(np.uint16)
    seeds = rng.integers(0, 2**63, R).astype(np.uint64)
    subs = rng.integers(0, 1000, R).astype(np.uint64)
    return p, hist, hoff, seeds, subs


def _check_logits(hidden, weight, logits):
    H = hidden.shape[1]
    h64 = hidden.double()
    w64 = weight.double()
    ref = h64 @ w64.T
    # Each output is at most H/32 sequential f32 additions per lane, a
    # 5-level butterfly and one rounding per product.
    bound = (h64.abs() @ w64.abs().T) * ((H // 32 + 8) * 2.0 ** -24)
    err = (logits.double() - ref).abs()
    assert bool((err <= bound + 1e-30).all()), float((err - bound).max())


@pytest.mark.parametrize("R,V,H,hdt,talker", [
    (1, 3072, 1024, torch.bfloat16, True),
    (16, 3072, 1024, torch.float32, True),
    (5, 2048, 1024, torch.bfloat16, False),
    (3, 2048, 2048, torch.float32, False),
])
def test_head_sample_matches_projection_and_sampler(R, V, H, hdt, talker):
    hidden, weight = _inputs(R, V, H, hdt, seed=R * 7 + V)
    p, hist, hoff, seeds, subs = _rows(R, V, seed=R + H, talker=talker)
    dp = torch.from_numpy(p.view(np.uint8).copy()).to(DEV)
    ds = torch.from_numpy(seeds.view(np.int64)).to(DEV)
    du = torch.from_numpy(subs.view(np.int64)).to(DEV)
    kw = {}
    if talker:
        kw = {"history": torch.from_numpy(hist.view(np.int16)).to(DEV),
              "history_offsets": torch.from_numpy(hoff).to(DEV)}
    for call in range(2):  # two calls in a row: the completion counter resets
        tok, st, logits = q3s.head_sample(hidden, weight, dp, ds, du, **kw)
        torch.cuda.synchronize()
        _check_logits(hidden, weight, logits)
        t2, s2 = q3s.sample_batch(logits, dp, ds, du, **kw)
        torch.cuda.synchronize()
        assert torch.equal(tok, t2) and torch.equal(st, s2), call
        x = logits.cpu().numpy().reshape(-1)
        off = np.arange(R, dtype=np.int64) * V
        voc = np.full(R, V, np.int32)
        ref = oracle.sample_rows(x, off, voc, p, seeds, subs, hist if talker else None,
                                 hoff if talker else None)
        np.testing.assert_array_equal(st.cpu().numpy(), ref["status"])
        np.testing.assert_array_equal(tok.cpu().numpy().view(np.uint32), ref["tokens"])


def test_head_sample_rejects_bad_shapes():
    hidden, weight = _inputs(17, 2048, 1024, torch.float32, seed=1)
    p = q3s.make_params(1, top_k=50)
    z = torch.zeros(17, dtype=torch.int64, device=DEV)
    with pytest.raises(q3s.LibraryError):
        q3s.head_sample(hidden, weight, p, z, z)            # more than 16 rows
    h2 = torch.zeros((2, 1020), device=DEV)
    w2 = torch.zeros((2048, 1020), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(q3s.LibraryError):
        q3s.head_sample(h2, w2, p, z[:2], z[:2])            # H not a multiple of 8


@pytest.mark.parametrize("hdt,pad", [(torch.bfloat16, 4), (torch.float32, 1)])
def test_head_sample_unaligned_hidden_rows(hdt, pad):
    """Hidden rows that do not start on 16-byte boundaries (a padded row
    stride) are staged element by element: the same logits and ids as the
    contiguous rows, which are staged with 16-byte loads."""
    R, V, H = 6, 3072, 1024
    hidden, weight = _inputs(R, V, H, hdt, seed=91)
    wide = torch.zeros((R, H + pad), dtype=hdt, device=DEV)
    wide[:, :H] = hidden
    view = wide[:, :H]
    assert view.stride(0) == H + pad
    p, hist, hoff, seeds, subs = _rows(R, V, seed=92, talker=True)
    dp = torch.from_numpy(p.view(np.uint8).copy()).to(DEV)
    ds = torch.from_numpy(seeds.view(np.int64)).to(DEV)
    du = torch.from_numpy(subs.view(np.int64)).to(DEV)
    kw = {"history": torch.from_numpy(hist.view(np.int16)).to(DEV),
          "history_offsets": torch.from_numpy(hoff).to(DEV)}
    a = q3s.head_sample(hidden, weight, dp, ds, du, **kw)
    b = q3s.head_sample(view, weight, dp, ds, du, **kw)
    torch.cuda.synchronize()
    assert torch.equal(a[2], b[2])
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    _check_logits(hidden, weight, b[2])
