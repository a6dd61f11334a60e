"""Continuous batching of sessions (q3s_scheduler_*), checked against each
session replayed alone with the oracle (its own Sampler, its own c0
history, the reference's call order of talker.rs:500-566 and
code_predictor.rs:337-427).  The gates are the reference's plan for this
scheduler (tasks/P12-c-abi-and-continuous-batching.md): concurrent sessions
stay isolated, and batching leaves every session's deterministic output
unchanged, while sessions join, leave and fail between frames.

Bar: codes, statuses, counters and histories exact.
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
G = 16
TALKER_V, CP_V = 3072, 2048


def logits_for(sid, frame, group):
    """A session's logits for one step, independent of who else is batched."""
    rng = np.random.default_rng([sid, frame, group])
    if group == 0:
        return (rng.standard_normal(TALKER_V) * 2.5).astype(np.float32)
    return (rng.standard_normal(CP_V) * 3.0).astype(np.float32)


class Session:
    """A session's configuration and its oracle replay (the session alone)."""

    def __init__(self, sid, seed, talker, predictor, talker_do_sample=True,
                 predictor_do_sample=True, history=()):
        self.sid, self.seed = sid, seed
        self.talker, self.predictor = talker, predictor
        self.tds, self.pds = talker_do_sample, predictor_do_sample
        self.history = [int(h) for h in history]
        self.o = oracle.OracleSampler(seed)
        self.stopped = 0

    def add_to(self, sched):
        sched.add(self.sid, self.seed, self.talker, self.predictor,
                  talker_do_sample=self.tds, predictor_do_sample=self.pds,
                  suppress_from=2048, allow_token=2150, history=self.history)

    def replay_frame(self, frame):
        """(codes, status) the session gets alone in this frame."""
        codes = []
        for g in range(G):
            row = logits_for(self.sid, frame, g)
            o = self.talker if g == 0 else self.predictor
            d = {"temperature": o.temperature, "top_k": o.top_k, "top_p": o.top_p,
                 "repetition_penalty": o.repetition_penalty}
            if g == 0:
                st, tok = self.o.sample_with_mode(row, d, self.tds, 2048, 2150, self.history)
            else:
                st, tok = self.o.sample_with_mode(row, d, self.pds, None, None, [])
            if st:
                self.stopped = st
                return codes, st
            codes.append(tok)
            if g == 0:
                self.history.append(tok)
        return codes, 0


def run_frame(sched, frame):
    ids = sched.begin_frame()
    for g in range(G):
        x = np.stack([logits_for(sid, frame, g) for sid in ids]) if ids else \
            np.zeros((0, TALKER_V if g == 0 else CP_V), np.float32)
        sched.step(g, torch.from_numpy(x).to(DEV))
    codes, status = sched.end_frame()
    return ids, codes, status


def make_sessions():
    T = q3s.SamplingOptions
    rng = np.random.default_rng(3)
    s = []
    for i in range(8):
        talker = T(0.9, 50, 1.0, 1.05)
        pred = T(0.9, 50, 1.0, 1.0)
        if i == 1:
            talker = T(0.7, 0, 0.8, 1.1)         # nucleus path with a penalty
        if i == 3:
            pred = T(1.0, 200, 0.9, 1.0)         # top-k then top-p
        hist = rng.integers(0, 2048, rng.integers(0, 400))
        s.append(Session(100 + i, int(rng.integers(0, 2**63)), talker, pred,
                         talker_do_sample=(i != 5), predictor_do_sample=(i != 6),
                         history=hist))
    s[4].talker = T(0.9, 50, 1.5, 1.05)           # invalid top_p: fails at its first call
    return s


def test_sessions_are_isolated_and_batching_keeps_their_output():
    sessions = make_sessions()
    sched = q3s.Scheduler(max_sessions=8, groups=G, history_capacity=1024)
    for s in sessions[:6]:
        s.add_to(sched)
    for frame in range(4):
        if frame == 1:
            for s in sessions[6:]:
                s.add_to(sched)
        if frame == 2:
            sched.cancel(sessions[2].sid)
            sessions[2].stopped = -1
        ids, codes, status = run_frame(sched, frame)
        expect_active = [s for s in sessions
                         if s.stopped == 0 and (frame >= 1 or s.sid < 106)]
        assert sorted(ids) == sorted(s.sid for s in expect_active), frame
        by_id = {s.sid: s for s in sessions}
        for r, sid in enumerate(ids):
            s = by_id[sid]
            want, st = s.replay_frame(frame)
            assert status[r] == st, (frame, sid)
            assert codes[r, :len(want)].tolist() == want, (frame, sid)
            if st == 0:
                sub, hist = sched.session_state(sid)
                assert sub == s.o.subsequence_counter, (frame, sid)
                assert hist == s.history, (frame, sid)
        np.testing.assert_array_equal(sched.codes_device().cpu().numpy().view(np.uint32), codes)
    assert sessions[4].stopped == q3s.STATUS_INVALID_TOP_P
    assert sessions[4].sid not in sched.active
    sched.close()


def test_one_session_alone_matches_the_batched_run():
    """The same session alone in its own scheduler and batched with seven
    others: identical codes and counters frame by frame."""
    sessions = make_sessions()
    batched = q3s.Scheduler(max_sessions=8, groups=G, history_capacity=1024)
    alone = q3s.Scheduler(max_sessions=1, groups=G, history_capacity=1024)
    for s in sessions:
        s.add_to(batched)
    sessions[1].add_to(alone)
    for frame in range(3):
        ids, codes, status = run_frame(batched, frame)
        ids1, codes1, status1 = run_frame(alone, frame)
        r = ids.index(sessions[1].sid)
        assert ids1 == [sessions[1].sid]
        assert status[r] == status1[0] == 0
        np.testing.assert_array_equal(codes[r], codes1[0])
        assert batched.session_state(sessions[1].sid) == alone.session_state(sessions[1].sid)
    batched.close()
    alone.close()


def test_scheduler_rejects_misuse():
    T = q3s.SamplingOptions
    sched = q3s.Scheduler(max_sessions=2, groups=G, history_capacity=8)
    o = T(0.9, 50, 1.0, 1.0)
    sched.add(1, 7, o, o)
    with pytest.raises(q3s.LibraryError):
        sched.add(1, 8, o, o)                       # duplicate id
    with pytest.raises(q3s.LibraryError):
        sched.add(2, 8, o, o, history=range(9))     # longer than the capacity
    sched.add(2, 8, o, o)
    with pytest.raises(q3s.LibraryError):
        sched.add(3, 9, o, o)                       # all slots in use
    with pytest.raises(q3s.LibraryError):
        sched.cancel(42)                            # unknown session
    ids = sched.begin_frame()
    assert sorted(ids) == [1, 2]
    x = torch.zeros((2, TALKER_V), device=DEV)
    with pytest.raises(q3s.LibraryError):
        sched.step(1, torch.zeros((2, CP_V), device=DEV))   # groups out of order
    sched.step(0, x)
    with pytest.raises(q3s.LibraryError):
        sched.end_frame()                           # groups left
    with pytest.raises(q3s.LibraryError):
        sched.begin_frame()                         # frame still open
    for g in range(1, G):
        sched.step(g, torch.zeros((2, CP_V), device=DEV))
    codes, status = sched.end_frame()
    assert status.tolist() == [0, 0]
    sched.cancel(1)
    assert sched.begin_frame() == [2]
    sched.close()


def test_capacity_counts_a_cancelled_failed_session_once():
    """A session that fails in a frame and is also cancelled frees one slot:
    with two slots, one session staying and that one leaving, one add fits
    and a second is refused."""
    T = q3s.SamplingOptions
    sched = q3s.Scheduler(max_sessions=2, groups=G, history_capacity=8)
    o = T(0.9, 50, 1.0, 1.0)
    sched.add(1, 7, o, o)
    sched.add(2, 8, T(0.9, 50, 1.5, 1.0), o)       # invalid top_p: fails at its first call
    ids, codes, status = run_frame(sched, 0)
    assert dict(zip(ids, status.tolist()))[2] == q3s.STATUS_INVALID_TOP_P
    sched.cancel(2)
    sched.add(3, 9, o, o)
    with pytest.raises(q3s.LibraryError):
        sched.add(4, 10, o, o)
    assert sorted(sched.begin_frame()) == [1, 3]
    for g in range(G):
        sched.step(g, torch.zeros((2, TALKER_V if g == 0 else CP_V), device=DEV))
    sched.end_frame()
    sched.close()
