"""ORACLE — test infrastructure only.

Exactness report of the device sampler against the reference sampler as it
runs on Linux: src/talker/sampling.rs computes every exponential with Rust's
f32::exp (sampling.rs:673, 685, 712), which calls the platform libm expf
(glibc here).  The device kernel uses a correctly rounded exp, which agrees
with glibc's expf except on a few inputs (one ulp apart).  This module runs
the oracle in its glibc mode (oracle.EXP_LIBM) on the same rows and counts
where and why the two differ:

  * statuses (and so Philox consumption) must be identical on every row;
  * the candidate and top-k masks (bits 0 and 1) involve no exp and must be
    identical;
  * the top-p mask (bit 2) may differ only on rows whose nucleus decision lies
    within `tol` of top_p (`topp_gap`, sampling.rs:690-697);
  * token ids may differ only on rows whose Philox uniform lies within `tol`
    of a CDF boundary of the final draw (`boundary_gap`, sampling.rs:720-728)
    or whose nucleus decision does;
  * final probabilities agree within `prob_rtol` relative wherever the masks
    agree.

Imported only by tests/ and by bench.py outside its timed region, as the
checker.
"""
from __future__ import annotations

import numpy as np

import oracle

TOL = 1e-6
PROB_RTOL = 1e-5


def libm_report(layout, got_tokens, got_status, *, sample=None, got_probs=None, got_masks=None,
                tol: float = TOL, prob_rtol: float = PROB_RTOL, nthreads: int = 1) -> dict:
    """Compares device results with the glibc-expf oracle.

    layout: the tuple of Workload.oracle_layout() (all rows of the check).
    got_tokens / got_status: device outputs for those rows.
    sample: indices (into those rows) whose device debug outputs
    got_probs / got_masks ([len(sample), max vocab]) are compared too.
    Returns counts; `violations` is 0 when every difference is explained by a
    boundary row as described in the module docstring.
    """
    logits, offsets, vocab, params, seeds, subseqs, hist, hoff = layout
    ref = oracle.sample_rows(logits, offsets, vocab, params, seeds, subseqs, hist, hoff,
                             exp_mode=oracle.EXP_LIBM, nthreads=nthreads)
    got_tokens = np.asarray(got_tokens).view(np.uint32)
    got_status = np.asarray(got_status)
    status_diff = got_status != ref["status"]
    ok = (ref["status"] == 0) & ~status_diff
    draw_b = ok & (ref["boundary_gap"] < tol)
    topp_b = ok & (ref["topp_gap"] < tol)
    boundary = draw_b | topp_b
    tok_diff = ok & (got_tokens != ref["tokens"])
    rep = {
        "rows": int(got_status.size),
        "ok_rows": int(ok.sum()),
        "status_mismatch_rows": int(status_diff.sum()),
        "boundary_rows": int(boundary.sum()),
        "draw_boundary_rows": int(draw_b.sum()),
        "topp_boundary_rows": int(topp_b.sum()),
        "libm_mismatch_rows": int(tok_diff.sum()),
        "unexplained_mismatch_rows": int((tok_diff & ~boundary).sum()),
    }
    violations = rep["status_mismatch_rows"] + rep["unexplained_mismatch_rows"]
    if sample is not None and got_probs is not None:
        sample = np.asarray(sample)
        sub = _subset(layout, sample)
        rs = oracle.sample_rows(*sub, exp_mode=oracle.EXP_LIBM, want_probs=True,
                                nthreads=nthreads)
        mask_hard = mask_topp = prob_bad = 0
        worst = 0.0
        sub_vocab = sub[2]
        for j, r in enumerate(sample):
            if rs["status"][j] != 0 or got_status[r] != 0:
                continue
            n = int(sub_vocab[j])
            gm = np.asarray(got_masks[j, :n])
            wm = rs["masks"][j, :n]
            if np.any((gm & 3) != (wm & 3)):
                mask_hard += 1
            if np.any((gm & 4) != (wm & 4)):
                mask_topp += 1
                if not topp_b[r]:
                    violations += 1
                continue
            gp = np.asarray(got_probs[j, :n], np.float64)
            wp = rs["probs"][j, :n].astype(np.float64)
            nz = wp != 0
            if np.any((gp != 0) != nz):
                prob_bad += 1
                continue
            if nz.any():
                rel = np.abs(gp[nz] - wp[nz]) / np.abs(wp[nz])
                m = float(rel.max())
                worst = max(worst, m)
                if m > prob_rtol:
                    prob_bad += 1
        rep.update({"masked_rows_compared": int(sample.size),
                    "topk_mask_mismatch_rows": mask_hard,
                    "topp_mask_mismatch_rows": mask_topp,
                    "prob_mismatch_rows": prob_bad,
                    "max_prob_rel_diff": worst})
        violations += mask_hard + prob_bad
    rep["violations"] = int(violations)
    return rep


def _subset(layout, idx):
    """The oracle layout of rows `idx` of `layout` (re-based offsets)."""
    logits, offsets, vocab, params, seeds, subseqs, hist, hoff = layout
    parts = [logits[int(offsets[r]): int(offsets[r]) + int(vocab[r])] for r in idx]
    v = vocab[idx].astype(np.int32)
    off = np.zeros(idx.size, np.int64)
    off[1:] = np.cumsum(v[:-1].astype(np.int64))
    p = params[idx] if params.size > 1 else params
    h = ho = None
    if hoff is not None:
        chunks = [hist[hoff[r]:hoff[r + 1]] for r in idx]
        ho = np.zeros(idx.size + 1, np.int64)
        ho[1:] = np.cumsum([c.size for c in chunks])
        h = np.concatenate(chunks) if chunks else np.zeros(0, np.uint16)
    return (np.concatenate(parts) if parts else np.zeros(1, np.float32), off, v, p,
            seeds[idx], subseqs[idx], h, ho)
