"""q3s_sample_batch_static (the entry point for callers that must not
allocate device memory during generation, e.g. engines whose device memory
belongs to their own pool allocator; its workspace is a file-scope device
array) against q3s_sample_batch (the context-allocated workspace) on the
same inputs, through the C ABI, two calls in a row so the second call runs
on the workspace the first one left behind.

Bar: tokens and statuses exact, final probabilities within 1e-5 relative and
masks exact.  This file sorts last so it also runs after every other GPU test
in one process; it passes alone in a fresh process as well.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes
    pytest.skip("needs a CUDA device", allow_module_level=True)

import q3s  # noqa: E402
from q3s import workloads  # noqa: E402

DEV = torch.device("cuda:0")
PROB_RTOL = 1e-5


def _both(w, ctx):
    """(context-workspace result, static-workspace result) with debug outputs."""
    args = w.device_args(DEV)
    params, seeds, subseqs = args.pop("params"), args.pop("seeds"), args.pop("subseqs")
    ref = q3s.sample_batch(w.logits, params, seeds, subseqs, debug=True, ctx=ctx, **args)
    got = q3s.sample_batch_static(w.logits, params, seeds, subseqs, debug=True, ctx=ctx, **args)
    torch.cuda.synchronize()
    return ref, got


def _assert_same(ref, got, w, label):
    rt, rs, rp, rm = (x.cpu().numpy() for x in ref)
    gt, gs, gp, gm = (x.cpu().numpy() for x in got)
    np.testing.assert_array_equal(gs, rs, err_msg=f"{label}: status")
    np.testing.assert_array_equal(gt, rt, err_msg=f"{label}: tokens")
    # The debug outputs are defined over each row's own vocabulary only.
    n = np.full(w.num_rows, w.vocab) if w.row_vocab is None else w.row_vocab
    inside = np.arange(rm.shape[1])[None, :] < np.asarray(n)[:, None]
    np.testing.assert_array_equal(gm[inside], rm[inside], err_msg=f"{label}: masks")
    np.testing.assert_allclose(gp[inside], rp[inside], rtol=PROB_RTOL, atol=0,
                               err_msg=f"{label}: probs")


def test_static_workspace_matches_context_workspace_two_calls():
    ctx = q3s.Context(0)
    # Call 1: every row on the general path (top-k off, top-p 0.8, penalty),
    # which is the path that uses the workspace.
    w1 = workloads.talker_batch(DEV, rows=1024)
    ref1, got1 = _both(w1, ctx)
    assert int((ref1[1] == 0).sum()) == w1.num_rows
    _assert_same(ref1, got1, w1, "talker_batch")
    # Call 2: a mixed batch (fast and general rows, two row lengths) on the
    # workspace call 1 left behind.
    w2 = workloads.hetero(DEV, streams=128)
    ref2, got2 = _both(w2, ctx)
    _assert_same(ref2, got2, w2, "hetero")
    ctx.close()


def test_static_call_allocates_no_device_memory():
    ctx = q3s.Context(0)
    w = workloads.talker_batch(DEV, rows=512)
    args = w.device_args(DEV)
    params, seeds, subseqs = args.pop("params"), args.pop("seeds"), args.pop("subseqs")
    out = (torch.empty(w.num_rows, dtype=torch.int32, device=DEV),
           torch.empty(w.num_rows, dtype=torch.uint8, device=DEV))
    ref_t, ref_s = q3s.sample_batch(w.logits, params, seeds, subseqs, ctx=ctx, **args)
    # The first call on the device does the set-up (symbol lookup).
    q3s.sample_batch_static(w.logits, params, seeds, subseqs, ctx=ctx, out=out, **args)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info(DEV)[0]
    q3s.sample_batch_static(w.logits, params, seeds, subseqs, ctx=ctx, out=out, **args)
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info(DEV)[0]
    assert free_after >= free_before
    assert torch.equal(out[0], ref_t) and torch.equal(out[1], ref_s)
    ctx.close()


def test_static_rejects_vocab_beyond_maximum():
    ctx = q3s.Context(0)
    V = q3s.MAX_VOCAB + 32
    logits = torch.zeros((2, V), dtype=torch.float32, device=DEV)
    params = q3s.make_params(1, top_k=50)
    seeds = torch.zeros(2, dtype=torch.int64, device=DEV)
    with pytest.raises(q3s.LibraryError, match="exceeds the static-workspace maximum"):
        q3s.sample_batch_static(logits, params, seeds, seeds, ctx=ctx)
    ctx.close()
