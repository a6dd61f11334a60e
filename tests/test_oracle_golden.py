"""Pins the oracle (CPU restatement of src/talker/sampling.rs) to the
reference's own golden vectors and unit-test literals.  CPU only."""
import math
import subprocess

import numpy as np
import pytest

import golden_io as gio

SAMPLE_OPTS = {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0}


def test_philox_fixture_words_and_uniform_bits(oracle_mod):
    # fixtures/alignment/p02_philox_vectors.json and sampling.rs:931-985.
    for case in gio.load("philox.json")["cases"]:
        seed = int(case["seed"])
        for s in case["samples"]:
            sub = int(s["subsequence"])
            ctr = [case["ctr_lo"], 0, sub & 0xFFFFFFFF, sub >> 32]
            words = oracle_mod.philox4x32_10(ctr, seed & 0xFFFFFFFF, seed >> 32)
            assert words == s["words"], case["name"]
            u = oracle_mod.next_uniform(seed, sub, case["ctr_lo"])
            assert gio.f32_bits(u) == s["uniform_bits"], case["name"]


def test_uniform_range_endpoints(oracle_mod):
    # u = ((w0 as f32) + 0.5) * 2^-32 lies in (0, 1] (sampling.rs:373).
    us = np.array([oracle_mod.next_uniform(7, s) for s in range(2000)], dtype=np.float32)
    assert (us > 0).all() and (us <= 1).all()


def test_cr_expf_matches_binary64_exp_on_random_inputs(oracle_mod):
    rng = np.random.default_rng(1)
    xs = np.concatenate([
        -rng.uniform(0, 104, 20000), -rng.uniform(0, 1e-3, 2000), -rng.uniform(0, 20, 20000),
        np.array([0.0, -0.0, -87.3, -103.9, -103.97, -104.0, 1.0, 10.0, 88.7, 88.73, 89.0]),
    ]).astype(np.float32)
    for x in xs:
        ref = np.float32(math.exp(float(x))) if float(x) > -746 else np.float32(0.0)
        got = np.float32(oracle_mod.cr_expf(float(x)))
        assert got.view(np.uint32) == ref.view(np.uint32), float(x)
    assert oracle_mod.cr_expf(float("-inf")) == 0.0
    assert math.isinf(oracle_mod.cr_expf(float("inf")))
    assert math.isnan(oracle_mod.cr_expf(float("nan")))


def test_cr_expf_exhaustive_slice():
    """Every binary32 in [-1/16, -0] (67M inputs) against long double expl;
    `oracle/expf_exhaustive` without arguments covers all of [-104, -0]."""
    import oracle
    exe = oracle.HERE / "expf_exhaustive"
    if not exe.exists():
        subprocess.run(["make", "-s", "-C", str(oracle.HERE), str(exe)], check=True)
    out = subprocess.run([str(exe), "80000000", "BD800000"], capture_output=True, text=True,
                         check=True).stdout
    assert "cr_mismatch=0" in out, out


def test_repetition_penalty_fixture(oracle_mod):
    # fixtures/alignment/p02_repetition_penalty_vectors.json via
    # tests/repetition_penalty_test.rs:266-327 and :329-422.
    for case in gio.load("repetition_penalty.json")["cases"]:
        logits = np.array([gio.bits_to_f32(b) for b in case["logit_bits"]], dtype=np.float32)
        opts = case["options"]
        sf, allow = case["suppress_from"], case["allow_suppressed_token"]
        # Candidate order and bits before/after the penalty and the temperature.
        def cand(vals):
            idx = [i for i, v in enumerate(vals) if np.isfinite(v) and
                   (sf is None or i < sf or i == allow)]
            return sorted(idx, key=lambda i: (-float(vals[i]), i))
        before = cand(logits)
        assert before == case["candidates_before_repetition"], case["name"]
        assert [gio.f32_bits(logits[i]) for i in before] == case["candidates_before_repetition_bits"]
        if opts["temperature"] > 0:
            after = oracle_mod.apply_repetition_penalty(logits, case["history"],
                                                        opts["repetition_penalty"])
        else:
            after = logits.copy()
        order = cand(after)
        assert order == case["candidates_after_repetition"], case["name"]
        assert [gio.f32_bits(after[i]) for i in order] == case["after_repetition_bits"], case["name"]
        if opts["temperature"] > 0:
            inv = np.float32(1.0) / np.float32(opts["temperature"])
            scaled = [gio.f32_bits(np.float32(after[i]) * inv) for i in order]
        else:
            scaled = [gio.f32_bits(after[i]) for i in order]
        assert scaled == case["after_temperature_bits"], case["name"]
        # The Sampler replay: sample draws with subsequences 0, 1, 2, ...
        s = oracle_mod.OracleSampler(int(case["seed"]))
        for k, sample in enumerate(case["samples"]):
            st, tok = s.sample(logits, opts, sf, allow, case["history"])
            assert st == oracle_mod.OK and tok == sample["expected"], (case["name"], k)
            if sample["uniform_bits"] is not None:
                u = oracle_mod.next_uniform(int(case["seed"]), k)
                assert gio.f32_bits(u) == sample["uniform_bits"]


def test_deterministic_token_sequences_fixture(oracle_mod):
    # tests/deterministic_token_sequence_test.rs:52-98 over 12 cases / 233 calls.
    data = gio.load("token_sequences.json")
    ncalls = 0
    for case in data["cases"]:
        s = oracle_mod.OracleSampler(case["seed"])
        frames: dict = {}
        c0 = []
        for call in case["calls"]:
            assert s.subsequence_counter == call["subsequence"], case["id"]
            logits = gio.decode_row(call["logits"])
            o = call["options"]
            st, tok = s.sample_with_mode(logits, o, o["do_sample"], call["suppress_from"],
                                         call["allow_token"], call["history"])
            assert st == oracle_mod.OK and tok == call["expected"], (case["id"], call["codebook"])
            if call["frame"] < len(case["frames"]):
                frames.setdefault(call["frame"], []).append(tok)
                if call["codebook"] == 0:
                    c0.append(tok)
            ncalls += 1
        assert [frames[k] for k in sorted(frames)] == case["frames"], case["id"]
        assert c0 == case["c0_history"], case["id"]
        assert s.subsequence_counter == case["draw_count"], case["id"]
        assert s.diagnostics()["sequence_len"] == min(64, len(case["calls"]))
    assert ncalls == 233


def test_suppression_eos_fixture(oracle_mod):
    # tests/suppression_eos_test.rs:52-75: greedy_select over ones(V) stays in
    # the allowed set; the allowed set equals the suppression mask.
    for case in gio.load("suppression_eos.json")["cases"]:
        v, sf, eos, step = case["vocab_size"], case["suppress_from"], case["eos"], case["step"]
        assert sf == v - 1024
        allowed = set()
        for lo, hi in case["allowed_ranges"]:
            allowed.update(range(lo, hi))
        assert (eos in allowed) == (step >= 2)
        allow = eos if step >= 2 else None
        st, tok = oracle_mod.greedy_select(np.ones(v, np.float32), sf, allow)
        assert st == oracle_mod.OK and tok in allowed
        r = oracle_mod.sample_logits(np.zeros(v, np.float32), SAMPLE_OPTS, sf, allow, [], 0.5)
        assert set(np.flatnonzero(r.masks & 1).tolist()) == allowed


def test_unit_test_literals(oracle_mod):
    data = gio.load("unit_literals.json")
    for case in data["cases"]:
        logits = gio.decode_row(case["logits"])
        if case["kind"] == "greedy_select":
            st, tok = oracle_mod.greedy_select(logits, case["suppress_from"], case["allow_token"])
            assert st == oracle_mod.OK and tok == case["expected"], case["name"]
            continue
        if case["uniform"] is None:  # a Sampler call (suppression_eos_test.rs:77-105)
            s = oracle_mod.OracleSampler(77)
            st, tok = s.sample_with_mode(logits, case["options"], True, case["suppress_from"],
                                         case["allow_token"], case["history"])
        else:
            r = oracle_mod.sample_logits(logits, case["options"], case["suppress_from"],
                                         case["allow_token"], case["history"], case["uniform"])
            st, tok = r.status, r.token
        assert st == oracle_mod.OK and tok == case["expected"], case["name"]
    pen = data["penalty_bits"]
    x = np.array([gio.bits_to_f32(b) for b in pen["logits"]], np.float32)
    out = oracle_mod.apply_repetition_penalty(x, pen["history"], pen["penalty"])
    assert [gio.f32_bits(v) for v in out] == pen["expected"]
    for f in data["failures"]:
        s = oracle_mod.OracleSampler(f["seed"])
        st, _ = s.sample_with_mode(gio.decode_row(f["logits"]), f["options"], f["do_sample"],
                                   f["suppress_from"], f["allow_token"], [])
        assert st != oracle_mod.OK, f["name"]
        assert s.subsequence_counter == 0, f["name"]


def test_python_oracle_cases(oracle_mod):
    # Seeded cases decided by the reference's tools/ Python oracle.
    for case in gio.load("python_oracle_cases.json")["cases"]:
        logits = gio.decode_q64(case["logits_q64"])
        o = case["options"]
        s = oracle_mod.OracleSampler(int(case["seed"]))
        s.subsequence_counter = int(case["subsequence"])
        st, tok = s.sample_with_mode(logits, o, o["do_sample"], case["suppress_from"],
                                     case["allow_token"], case["history"])
        if case["status"] == "ok":
            assert st == oracle_mod.OK and tok == case["expected"], case["id"]
        else:
            assert st in (oracle_mod.SUPPRESSION_NO_CANDIDATE, oracle_mod.NO_CANDIDATE), case["id"]
        advanced = (s.subsequence_counter - int(case["subsequence"])) % (1 << 64)
        assert advanced == (1 if case["drew"] else 0), case["id"]


def test_top_p_boundary_masks_tail(oracle_mod):
    # sampling.rs:902-928.
    full = dict(SAMPLE_OPTS)
    filt = dict(SAMPLE_OPTS, top_p=0.8)
    logits = np.array([0.0, 2.0, 1.0], np.float32)
    for seed in range(256):
        a, b = oracle_mod.OracleSampler(seed), oracle_mod.OracleSampler(seed)
        _, t_all = a.sample_with_mode(logits, full, True)
        _, t_kept = b.sample_with_mode(logits, filt, True)
        if t_all != t_kept:
            assert t_kept == 1
            return
    pytest.fail("top-p boundary never changed the sampled candidate")


def test_subsequence_rollover(oracle_mod):
    # sampling.rs:996-1025.
    seed = 0x0123456789ABCDEF
    s = oracle_mod.OracleSampler(seed)
    s.subsequence_counter = 2**64 - 1
    logits = np.zeros(2, np.float32)
    _, first = s.sample(logits, SAMPLE_OPTS)
    _, second = s.sample(logits, SAMPLE_OPTS)
    expect = lambda u: 0 if u <= 0.5 else 1  # noqa: E731
    assert first == expect(oracle_mod.next_uniform(seed, 2**64 - 1))
    assert second == expect(oracle_mod.next_uniform(seed, 0))
    assert s.subsequence_counter == 1


def test_shared_philox_order_and_history_diagnostics(oracle_mod):
    # tests/sampling_config_test.rs:201-252.
    logits = np.array([0.1, 0.9], np.float32)
    sampled = {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.5}
    for talker in (False, True):
        for sub in (False, True):
            s = oracle_mod.OracleSampler(7)
            assert s.sample_with_mode(logits, sampled, talker, history=[0])[0] == 0
            for _ in range(15):
                assert s.sample_with_mode(logits, sampled, sub)[0] == 0
            assert s.subsequence_counter == int(talker) + 15 * int(sub)
    opts = {"temperature": 0.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 2.0}
    s = oracle_mod.OracleSampler(9)
    st, tok = s.sample_with_mode(np.array([0.0, 2.0], np.float32), opts, False, history=[1])
    assert st == 0 and tok == 1
    st, _ = s.sample_with_mode(np.array([0.0, 2.0], np.float32), dict(opts, temperature=1.0), True)
    assert st == 0
    d = s.diagnostics()
    assert d["history_nonempty_calls"] == 1 and d["call_count"] == 2


def test_seed_rerun_and_change(oracle_mod):
    # tests/deterministic_token_sequence_test.rs:100-119.
    logits = np.array([0.0, 1.0, 2.0], np.float32)

    def run(seed):
        s = oracle_mod.OracleSampler(seed)
        return [s.sample_with_mode(logits, SAMPLE_OPTS, True)[1] for _ in range(12)]
    assert run(7) == run(7)
    assert run(7) != run(8)


def test_libm_exp_mode_replays_fixtures(oracle_mod):
    # The literal Rust-on-Linux restatement (glibc expf) also replays the
    # reference's token sequences.
    data = gio.load("token_sequences.json")
    for case in data["cases"]:
        s = oracle_mod.OracleSampler(case["seed"], exp_mode=oracle_mod.EXP_LIBM)
        for call in case["calls"]:
            o = call["options"]
            st, tok = s.sample_with_mode(gio.decode_row(call["logits"]), o, o["do_sample"],
                                         call["suppress_from"], call["allow_token"],
                                         call["history"])
            assert st == 0 and tok == call["expected"]
