"""The exactness report (oracle/exactness.py) on CPU: the oracle in its
correctly rounded mode stands in for the device kernel (which computes the
same operations), compared with the oracle in glibc-expf mode, the reference
sampler as Rust's f32::exp runs it on Linux (src/talker/sampling.rs:673, 685,
712).  A planted token mismatch on a row far from every boundary must be
reported as a violation."""
import numpy as np
import pytest

import oracle
import exactness
from q3s import workloads


def cr_run(layout, want_probs=False):
    return oracle.sample_rows(*layout, exp_mode=oracle.EXP_CR, want_probs=want_probs,
                              nthreads=oracle.cpu_count())


CASES = [
    ("talker_single", lambda: workloads.talker_single("cpu", steps=300)),
    ("cp_frame", lambda: workloads.cp_frame("cpu", streams=16)),
    ("talker_batch", lambda: workloads.talker_batch("cpu", rows=256)),
    ("bandwidth_k50", lambda: workloads.bandwidth("cpu", rows=512, top_k=50)),
    ("hetero", lambda: workloads.hetero("cpu", streams=32)),
]


@pytest.mark.parametrize("name,make", CASES, ids=[c[0] for c in CASES])
def test_cr_against_libm_is_explained(name, make):
    w = make()
    lay = w.oracle_layout()
    got = cr_run(lay)
    sample = np.arange(0, w.num_rows, max(1, w.num_rows // 64))
    sub = exactness._subset(lay, sample)
    dbg = cr_run(sub, want_probs=True)
    rep = exactness.libm_report(lay, got["tokens"], got["status"], sample=sample,
                                got_probs=dbg["probs"], got_masks=dbg["masks"],
                                nthreads=oracle.cpu_count())
    assert rep["violations"] == 0, rep
    assert rep["status_mismatch_rows"] == 0
    assert rep["topk_mask_mismatch_rows"] == 0
    assert rep["libm_mismatch_rows"] <= rep["boundary_rows"]


def test_planted_mismatch_is_a_violation():
    w = workloads.bandwidth("cpu", rows=256, top_k=50)
    lay = w.oracle_layout()
    got = cr_run(lay)
    ref = oracle.sample_rows(*lay, exp_mode=oracle.EXP_LIBM)
    far = np.flatnonzero((ref["status"] == 0) & (ref["boundary_gap"] > 1e-3))
    assert far.size > 0
    tokens = got["tokens"].copy()
    r = int(far[0])
    tokens[r] = (tokens[r] + 1) % 3072
    rep = exactness.libm_report(lay, tokens, got["status"])
    assert rep["unexplained_mismatch_rows"] == 1
    assert rep["violations"] == 1
    status = got["status"].copy()
    status[r] = 6
    rep = exactness.libm_report(lay, got["tokens"], status)
    assert rep["status_mismatch_rows"] == 1 and rep["violations"] >= 1


def test_topp_gap_is_reported():
    # A row whose nucleus decision sits exactly on top_p: two equal
    # probabilities 0.5 and top_p 0.5 (the second position's preceding
    # cumulative is exactly 0.5).
    r = oracle.sample_logits(np.array([0.0, 0.0, -50.0], np.float32),
                             {"temperature": 1.0, "top_k": 0, "top_p": 0.5,
                              "repetition_penalty": 1.0})
    assert r.status == 0
    assert r.topp_gap == 0.0
    r = oracle.sample_logits(np.array([0.0, 0.0], np.float32),
                             {"temperature": 1.0, "top_k": 0, "top_p": 1.0,
                              "repetition_penalty": 1.0})
    assert r.topp_gap == float("inf")
