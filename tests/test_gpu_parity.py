"""GPU parity: the CUDA sampler through its C ABI against the oracle (the CPU
restatement of src/talker/sampling.rs) and the reference's golden vectors.

Bar: tokens, statuses, Philox consumption, masks (candidate / top-k / top-p)
bit-exact; final probabilities within 1e-5 relative (they are computed with
the same correctly rounded operations, so they agree exactly in practice).
"""
import math

import numpy as np
import pytest

import golden_io as gio

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - collected on CPU boxes
    pytest.skip("needs a CUDA device", allow_module_level=True)

import q3s  # noqa: E402
from q3s import workloads  # noqa: E402
import oracle  # noqa: E402

DEV = torch.device("cuda:0")
PROB_RTOL = 1e-5


def opts(d) -> q3s.SamplingOptions:
    return q3s.SamplingOptions(d["temperature"], int(d["top_k"]), d["top_p"],
                               d["repetition_penalty"])


def cuda_f32(x) -> "torch.Tensor":
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(DEV)


# ---------------------------------------------------------------------------
# Golden vectors through the stateful Sampler (the drop-in surface).
# ---------------------------------------------------------------------------
def test_token_sequences_fixture_on_gpu():
    data = gio.load("token_sequences.json")
    for case in data["cases"]:
        s = q3s.Sampler(case["seed"])
        for call in case["calls"]:
            assert s.subsequence_counter() == call["subsequence"], case["id"]
            o = call["options"]
            tok = s.sample_with_mode(cuda_f32(gio.decode_row(call["logits"])), opts(o),
                                     o["do_sample"], call["suppress_from"], call["allow_token"],
                                     call["history"])
            assert tok == call["expected"], (case["id"], call["frame"], call["codebook"])
        assert s.subsequence_counter() == case["draw_count"], case["id"]
        assert s.diagnostics()["sequence_len"] == min(64, len(case["calls"]))


def test_repetition_fixture_on_gpu():
    for case in gio.load("repetition_penalty.json")["cases"]:
        logits = np.array([gio.bits_to_f32(b) for b in case["logit_bits"]], np.float32)
        s = q3s.Sampler(int(case["seed"]))
        for sample in case["samples"]:
            tok = s.sample(cuda_f32(logits), opts(case["options"]), case["suppress_from"],
                           case["allow_suppressed_token"], case["history"])
            assert tok == sample["expected"], case["name"]


def test_unit_literals_on_gpu():
    data = gio.load("unit_literals.json")
    for case in data["cases"]:
        logits = gio.decode_row(case["logits"])
        if case["kind"] == "greedy_select":
            assert q3s.greedy_select(cuda_f32(logits), case["suppress_from"],
                                     case["allow_token"]) == case["expected"]
            continue
        o = case["options"]
        if case["uniform"] is None:
            s = q3s.Sampler(77)
            tok = s.sample_with_mode(cuda_f32(logits), opts(o), True, case["suppress_from"],
                                     case["allow_token"], case["history"])
        else:
            p = q3s.make_params(1, temperature=o["temperature"] if o["temperature"] > 0 else 1.0,
                                top_k=o["top_k"], top_p=o["top_p"],
                                repetition_penalty=o["repetition_penalty"],
                                do_sample=1 if o["temperature"] > 0 else 0,
                                suppress_from=-1 if case["suppress_from"] is None
                                else case["suppress_from"],
                                allow_token=-1 if case["allow_token"] is None
                                else case["allow_token"])
            hist = np.array(case["history"], np.uint16)
            ht = torch.from_numpy(hist.view(np.int16)).to(DEV) if hist.size else \
                torch.zeros(1, dtype=torch.int16, device=DEV)
            hoff = torch.tensor([0, hist.size], dtype=torch.int64, device=DEV)
            x = cuda_f32(logits).view(1, -1)
            tokens, status = q3s.sample_batch(
                x, p, torch.zeros(1, dtype=torch.int64, device=DEV),
                torch.zeros(1, dtype=torch.int64, device=DEV), history=ht, history_offsets=hoff,
                uniform_override=torch.tensor([case["uniform"]], dtype=torch.float32,
                                              device=DEV))
            assert int(status.item()) == 0, case["name"]
            tok = int(tokens.item())
        assert tok == case["expected"], case["name"]
    for f in data["failures"]:
        s = q3s.Sampler(f["seed"])
        with pytest.raises(q3s.SamplingError):
            s.sample_with_mode(cuda_f32(gio.decode_row(f["logits"])), opts(f["options"]),
                               f["do_sample"], f["suppress_from"], f["allow_token"], [])
        assert s.subsequence_counter() == 0, f["name"]


def test_python_oracle_cases_on_gpu():
    for case in gio.load("python_oracle_cases.json")["cases"]:
        o = case["options"]
        s = q3s.Sampler(int(case["seed"]))
        s.set_subsequence_counter(int(case["subsequence"]))
        x = cuda_f32(gio.decode_q64(case["logits_q64"]))
        if case["status"] == "ok":
            tok = s.sample_with_mode(x, opts(o), o["do_sample"], case["suppress_from"],
                                     case["allow_token"], case["history"])
            assert tok == case["expected"], case["id"]
        else:
            with pytest.raises(q3s.SamplingError):
                s.sample_with_mode(x, opts(o), o["do_sample"], case["suppress_from"],
                                   case["allow_token"], case["history"])
        advanced = (s.subsequence_counter() - int(case["subsequence"])) % (1 << 64)
        assert advanced == (1 if case["drew"] else 0), case["id"]


def test_sampler_counter_contract_on_gpu():
    # sampling.rs:996-1025 (rollover) and tests/sampling_config_test.rs:201-252.
    seed = 0x0123456789ABCDEF
    s = q3s.Sampler(seed)
    s.set_subsequence_counter(2**64 - 1)
    o = q3s.SamplingOptions(1.0, 0, 1.0, 1.0)
    x = torch.zeros(2, dtype=torch.float32, device=DEV)
    first, second = s.sample(x, o), s.sample(x, o)
    assert first == (0 if oracle.next_uniform(seed, 2**64 - 1) <= 0.5 else 1)
    assert second == (0 if oracle.next_uniform(seed, 0) <= 0.5 else 1)
    assert s.subsequence_counter() == 1
    logits = torch.tensor([0.1, 0.9], dtype=torch.float32, device=DEV)
    sampled = q3s.SamplingOptions(1.0, 0, 1.0, 1.5)
    for talker in (False, True):
        for sub in (False, True):
            s = q3s.Sampler(7)
            s.sample_with_mode(logits, sampled, talker, history=[0])
            for _ in range(15):
                s.sample_with_mode(logits, sampled, sub)
            assert s.subsequence_counter() == int(talker) + 15 * int(sub)
    events = []
    s = q3s.Sampler(3)
    s.sample_with_transfer_observer(logits, sampled, observer=lambda *e: events.append(e))
    assert events == [(0, q3s.TRANSFER_SAMPLED_TOKEN, 1)]


def test_seed_rerun_and_change_on_gpu():
    logits = torch.tensor([0.0, 1.0, 2.0], dtype=torch.float32, device=DEV)
    o = q3s.SamplingOptions(1.0, 0, 1.0, 1.0)

    def run(seed):
        s = q3s.Sampler(seed)
        return [s.sample_with_mode(logits, o, True) for _ in range(12)]
    assert run(7) == run(7)
    assert run(7) != run(8)


# ---------------------------------------------------------------------------
# Random batches with edge cases: batch kernel vs oracle.
# ---------------------------------------------------------------------------
VOCABS = [0, 1, 2, 3, 5, 31, 32, 33, 63, 64, 100, 127, 128, 129, 255, 256, 257, 1000, 2048,
          2049, 3072, 4095, 4096]


def random_row(rng, n):
    kind = rng.integers(0, 9)
    if kind == 0:
        x = rng.standard_normal(n) * rng.choice([0.1, 1.0, 3.0, 30.0])
    elif kind == 1:
        x = rng.integers(-4, 5, n).astype(np.float64)  # many exact ties
    elif kind == 2:
        x = np.full(n, -np.inf)
        k = rng.integers(0, 4)
        if n:
            x[rng.integers(0, n, k)] = rng.standard_normal(k)
    elif kind == 3:
        x = rng.standard_normal(n)
        for v in (np.nan, np.inf, -np.inf):
            if n:
                x[rng.integers(0, n, rng.integers(0, 3))] = v
    elif kind == 4:
        x = rng.choice([-1, 1], n) * 10.0 ** rng.uniform(25, 38.5, n)
    elif kind == 5:
        x = np.full(n, rng.standard_normal())
    elif kind == 6:
        x = rng.choice([0.0, -0.0, 1.0, -1.0], n)
    elif kind == 7:
        x = rng.standard_normal(n)
        if n:
            x[rng.integers(0, n, 5)] += 8.0
    else:
        x = rng.standard_normal(n) * 1e-3  # flat: large top-p nucleus
    with np.errstate(over="ignore", invalid="ignore"):
        return x.astype(np.float32)


def random_params(rng, n):
    p = q3s.make_params(1)[0]
    p["do_sample"] = 1 if rng.random() < 0.85 else 0
    p["temperature"] = rng.choice([0.9, 1.0, 0.7, 0.5, 1.5, 3.0, 1e-3, 0.2, 1e-40, 1e39, 0.0,
                                   -1.0, np.nan, np.inf])
    p["top_k"] = rng.choice([0, 0, 1, 2, 5, 50, 200, 256, max(n - 1, 0), n, n + 5])
    p["top_p"] = rng.choice([1.0, 1.0, 0.9, 0.8, 0.5, 0.999999999999, 1e-9, 0.95, 1.1, 0.0,
                             np.nan])
    p["repetition_penalty"] = rng.choice([1.0, 1.0, 1.05, 1.5, 0.7, 1.0000000001, 2.0, 0.0,
                                          -1.0])
    if rng.random() < 0.4:
        p["suppress_from"] = rng.choice([0, max(n - 1, 0), n, n + 10, rng.integers(0, n + 1)])
        p["allow_token"] = rng.choice([-1, rng.integers(0, max(n, 1)), n + 3])
    return p


def run_both(rows, params, seeds, subseqs, histories, dtype=torch.float32, uniform=None,
             pad_front=0):
    """Packs rows back to back (arbitrary alignment) and runs GPU and oracle."""
    R = len(rows)
    vocab = np.array([r.size for r in rows], np.int32)
    offsets = np.zeros(R, np.int64)
    offsets[1:] = np.cumsum(vocab[:-1].astype(np.int64))
    offsets += pad_front
    flat = np.concatenate([np.zeros(pad_front, np.float32)] + list(rows)) \
        if R else np.zeros(1, np.float32)
    if flat.size == 0:
        flat = np.zeros(1, np.float32)
    xt = torch.from_numpy(flat).to(DEV)
    if dtype == torch.bfloat16:
        xt = xt.to(torch.bfloat16)
        host = xt.float().cpu().numpy()
    else:
        host = flat
    hoff = np.zeros(R + 1, np.int64)
    hoff[1:] = np.cumsum([len(h) for h in histories])
    hist = np.concatenate([np.asarray(h, np.uint16) for h in histories]) if hoff[-1] else \
        np.zeros(1, np.uint16)
    maxv = int(vocab.max()) if R else 0
    uo = None if uniform is None else torch.from_numpy(np.asarray(uniform, np.float32)).to(DEV)
    t, s, pr, mk = q3s.sample_batch(
        xt, params, torch.from_numpy(seeds.view(np.int64)).to(DEV),
        torch.from_numpy(subseqs.view(np.int64)).to(DEV),
        row_offsets=torch.from_numpy(offsets).to(DEV), row_vocab=torch.from_numpy(vocab).to(DEV),
        vocab=max(maxv, 1), history=torch.from_numpy(hist.view(np.int16)).to(DEV),
        history_offsets=torch.from_numpy(hoff).to(DEV), uniform_override=uo, debug=True)
    torch.cuda.synchronize()
    ref = oracle.sample_rows(host, offsets, vocab, params, seeds, subseqs, hist, hoff,
                             uniform_override=None if uniform is None else np.asarray(uniform,
                                                                                      np.float32),
                             want_probs=True)
    return (t.cpu().numpy().view(np.uint32), s.cpu().numpy(), pr.cpu().numpy(),
            mk.cpu().numpy(), ref, vocab)


def assert_same(got_t, got_s, got_p, got_m, ref, vocab, label=""):
    np.testing.assert_array_equal(got_s, ref["status"], err_msg=f"status {label}")
    ok = ref["status"] == 0
    np.testing.assert_array_equal(got_t[ok], ref["tokens"][ok], err_msg=f"tokens {label}")
    for r in np.flatnonzero(ok):
        n = int(vocab[r])
        np.testing.assert_array_equal(got_m[r, :n], ref["masks"][r, :n],
                                      err_msg=f"masks row {r} {label}")
        np.testing.assert_allclose(got_p[r, :n], ref["probs"][r, :n], rtol=PROB_RTOL, atol=0,
                                   err_msg=f"probs row {r} {label}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_edge_batches_match_oracle(dtype, seed):
    rng = np.random.default_rng(1000 + seed)
    rows, params, hists = [], [], []
    for _ in range(300):
        n = int(rng.choice(VOCABS))
        rows.append(random_row(rng, n))
        params.append(random_params(rng, n))
        hl = int(rng.choice([0, 0, 1, 5, 64, 300]))
        hists.append(rng.integers(0, n + 8, hl).astype(np.uint16))
    params = np.array(params, dtype=q3s.ROW_PARAMS_DTYPE)
    seeds = rng.integers(0, 2**63, len(rows)).astype(np.uint64)
    subseqs = rng.integers(0, 2**63, len(rows)).astype(np.uint64)
    got = run_both(rows, params, seeds, subseqs, hists, dtype=dtype, pad_front=int(seed))
    assert_same(*got, label=f"dtype={dtype} seed={seed}")


def test_forced_uniform_endpoints_match_oracle():
    rng = np.random.default_rng(7)
    rows = [random_row(rng, 64) for _ in range(64)]
    params = q3s.make_params(64, top_k=0)
    uni = np.array([1.0, np.float32(2.0**-33), 0.5, 0.25] * 16, np.float32)
    got = run_both(rows, params, np.zeros(64, np.uint64), np.zeros(64, np.uint64),
                   [[] for _ in rows], uniform=uni)
    assert_same(*got, label="forced uniform")


def test_large_nucleus_crosses_many_chunks():
    # Nearly flat rows: the top-p nucleus spans > 256 sorted entries.
    rng = np.random.default_rng(11)
    rows = [(rng.standard_normal(3072) * 1e-3).astype(np.float32) for _ in range(8)]
    rows += [np.zeros(4096, np.float32) for _ in range(2)]
    params = q3s.make_params(len(rows), top_k=0, top_p=0.9)
    got = run_both(rows, params, np.arange(len(rows), dtype=np.uint64),
                   np.zeros(len(rows), np.uint64), [[] for _ in rows])
    assert_same(*got, label="large nucleus")


# ---------------------------------------------------------------------------
# The five workload configurations at oracle-friendly sizes.
# ---------------------------------------------------------------------------
def compare_workload(w, rows=None):
    args = w.device_args(DEV)
    t, s, pr, mk = q3s.sample_batch(w.logits, args.pop("params"), args.pop("seeds"),
                                    args.pop("subseqs"), debug=True, **args)
    torch.cuda.synchronize()
    R = w.num_rows
    sel = np.arange(R) if rows is None else np.asarray(rows)
    logits, offsets, vocab, params, seeds, subseqs, hist, hoff = w.oracle_layout(sel)
    ref = oracle.sample_rows(logits, offsets, vocab, params, seeds, subseqs, hist, hoff,
                             want_probs=True, nthreads=oracle.cpu_count())
    got_t = t.cpu().numpy().view(np.uint32)[sel]
    got_s = s.cpu().numpy()[sel]
    got_p = pr.cpu().numpy()[sel]
    got_m = mk.cpu().numpy()[sel]
    assert_same(got_t, got_s, got_p, got_m, ref, vocab, label=w.name)
    near = int(np.sum(ref["boundary_gap"][ref["status"] == 0] < 1e-6))
    return near


def test_workload_talker_single():
    near = compare_workload(workloads.talker_single(DEV, steps=200))
    print("talker_single rows within 1e-6 of a CDF boundary:", near)


def test_workload_cp_frame_bf16():
    compare_workload(workloads.cp_frame(DEV))


def test_workload_talker_batch():
    compare_workload(workloads.talker_batch(DEV, rows=1024))


@pytest.mark.parametrize("k", [1, 50, 256])
def test_workload_bandwidth_sample(k):
    compare_workload(workloads.bandwidth(DEV, rows=4096, top_k=k))


def test_workload_hetero_sample():
    compare_workload(workloads.hetero(DEV, streams=128))


# ---------------------------------------------------------------------------
# Full-size checks (65536 x 3072): a row sample against the oracle plus
# properties every row must satisfy.
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("k", [1, 50, 256])
def test_full_size_bandwidth(k):
    w = workloads.bandwidth(DEV, rows=65536, top_k=k)
    args = w.device_args(DEV)
    t, s = q3s.sample_batch(w.logits, args.pop("params"), args.pop("seeds"),
                            args.pop("subseqs"), **args)
    t2, s2 = q3s.sample_batch(w.logits, *[a for a in (w.device_args(DEV)["params"],
                                                       w.device_args(DEV)["seeds"],
                                                       w.device_args(DEV)["subseqs"])])
    torch.cuda.synchronize()
    assert bool((s == 0).all())
    assert torch.equal(t, t2) and torch.equal(s, s2)  # deterministic
    x = w.logits
    picked = x.gather(1, t.long().view(-1, 1)).view(-1)
    kth = torch.topk(x, k, dim=1).values[:, k - 1]
    assert bool((picked >= kth).all())  # every token is inside its top-k set
    if k == 1:
        assert bool((picked == x.max(dim=1).values).all())
    rows = np.random.default_rng(k).choice(65536, 512, replace=False)
    rows.sort()
    logits, offsets, vocab, params, seeds, subseqs, hist, hoff = w.oracle_layout(rows)
    ref = oracle.sample_rows(logits, offsets, vocab, params, seeds, subseqs, hist, hoff,
                             nthreads=oracle.cpu_count())
    np.testing.assert_array_equal(t.cpu().numpy().view(np.uint32)[rows], ref["tokens"])


def test_hetero_production_kernel_matches_oracle():
    """The launch without debug outputs compiles its own kernel (no debug
    code on the hot path): check its tokens and statuses on a mixed batch
    (top-p, penalties, suppression, two vocabularies)."""
    w = workloads.hetero(DEV, streams=256)
    args = w.device_args(DEV)
    t, s = q3s.sample_batch(w.logits, args.pop("params"), args.pop("seeds"), args.pop("subseqs"),
                            **args)
    torch.cuda.synchronize()
    rows = np.sort(np.random.default_rng(7).choice(w.num_rows, 1024, replace=False))
    logits, offsets, vocab, params, seeds, subseqs, hist, hoff = w.oracle_layout(rows)
    ref = oracle.sample_rows(logits, offsets, vocab, params, seeds, subseqs, hist, hoff,
                             nthreads=oracle.cpu_count())
    np.testing.assert_array_equal(s.cpu().numpy()[rows], ref["status"])
    np.testing.assert_array_equal(t.cpu().numpy().view(np.uint32)[rows], ref["tokens"])


def test_full_size_hetero_sample():
    w = workloads.hetero(DEV, streams=4096)
    rows = np.sort(np.random.default_rng(5).choice(w.num_rows, 1024, replace=False))
    compare_workload(w, rows)


# ---------------------------------------------------------------------------
# Greedy kernels.
# ---------------------------------------------------------------------------
def test_greedy_batch_modes_match_oracle():
    rng = np.random.default_rng(3)
    for n in (1, 2, 5, 64, 1000, 2048, 3072):
        for trial in range(20):
            x = random_row(rng, n)
            sf = [None, 0, n // 2, n, n + 5][trial % 5]
            allow = [None, n - 1, 0, n + 2][trial % 4]
            xt = cuda_f32(x).view(1, -1)
            st, tok = oracle.greedy_select(x, sf, allow)
            tt, ss = q3s.greedy_batch(xt, sf, allow, q3s.GREEDY_SELECT)
            assert int(ss.item()) == (0 if st == 0 else q3s.STATUS_SUPPRESSION_NO_CANDIDATE)
            if st == 0:
                assert int(tt.item()) == tok
            want = oracle.greedy_select_on_device(x, sf, allow)
            got = q3s.greedy_select_on_device(xt, sf, allow)
            assert int(got.item()) == want, (n, trial)


# ---------------------------------------------------------------------------
# Bounded waits and concurrent streams.
# ---------------------------------------------------------------------------
def oracle_tokens(w):
    lay = w.oracle_layout()
    return oracle.sample_rows(*lay, nthreads=oracle.cpu_count())


def test_bounded_stage_wait_gives_up_and_context_stays_usable():
    """With the ring refills held back, every row after a stage's first one
    waits for a generation that is never issued (no copy is in flight): the
    wait runs out after 2 ms, the row and the rest of its block end
    NOT_RUN, and the call returns.  The same context then samples normally."""
    R = 4096
    w = workloads.bandwidth(DEV, rows=R, top_k=50)
    ref = oracle_tokens(w)
    ctx = q3s.Context(0)
    a = w.device_args(DEV)
    p, s, u = a.pop("params"), a.pop("seeds"), a.pop("subseqs")
    ctx.set_test_hooks(stage_wait_ns=2_000_000, hold_refill=True)
    t, st = q3s.sample_batch(w.logits, p, s, u, ctx=ctx)
    torch.cuda.synchronize()
    st = st.cpu().numpy()
    t = t.cpu().numpy().view(np.uint32)
    assert set(np.unique(st).tolist()) <= {q3s.STATUS_OK, 255}
    grid = min((R + 15) // 16, torch.cuda.get_device_properties(DEV).multi_processor_count)
    ticket = np.arange(R) // grid  # row = block + ticket * grid
    assert np.all(st[ticket >= 8] == 255)  # every refill-dependent row gave up
    ok = st == q3s.STATUS_OK
    assert ok.sum() >= 1
    np.testing.assert_array_equal(t[ok], ref["tokens"][ok])
    ctx.set_test_hooks(0, False)
    t2, st2 = q3s.sample_batch(w.logits, p, s, u, ctx=ctx)
    torch.cuda.synchronize()
    assert bool((st2 == 0).all())
    np.testing.assert_array_equal(t2.cpu().numpy().view(np.uint32), ref["tokens"])


def _general_rows(seed):
    """The 1024-row talker batch with top-p 1: top-k off and no nucleus, so
    every row takes the general path and its per-warp global workspace."""
    w = workloads.talker_batch(DEV, rows=1024, seed=seed)
    w.params["top_p"] = 1.0
    return w


def test_general_path_rows_on_two_streams_of_one_context():
    """Rows on the general path use the per-stream workspace; two streams of
    one context run them concurrently and both match the oracle."""
    ctx = q3s.Context(0)
    ws = [_general_rows(2), _general_rows(12)]
    stats = torch.zeros(2 * len(q3s.PATH_NAMES), dtype=torch.int64, device=DEV)
    a = ws[0].device_args(DEV)
    ctx.set_path_stats(stats)
    q3s.sample_batch(ws[0].logits, a.pop("params"), a.pop("seeds"), a.pop("subseqs"), ctx=ctx,
                     **a)
    torch.cuda.synchronize()
    ctx.set_path_stats(None)
    assert q3s.path_report(stats) .keys() == {"general_rules"}
    refs = [oracle_tokens(w) for w in ws]
    streams = [torch.cuda.Stream(DEV), torch.cuda.Stream(DEV)]
    args = []
    for w in ws:
        a = w.device_args(DEV)
        args.append((a.pop("params"), a.pop("seeds"), a.pop("subseqs"), a))
    torch.cuda.synchronize()
    outs = [None, None]
    for _ in range(6):
        for i in range(2):
            p, s, u, a = args[i]
            with torch.cuda.stream(streams[i]):
                outs[i] = q3s.sample_batch(ws[i].logits, p, s, u, ctx=ctx,
                                           stream=streams[i].cuda_stream, **a)
    torch.cuda.synchronize()
    for i in range(2):
        t, st = outs[i]
        np.testing.assert_array_equal(st.cpu().numpy(), refs[i]["status"])
        np.testing.assert_array_equal(t.cpu().numpy().view(np.uint32), refs[i]["tokens"])


def test_path_stats_count_every_row_once():
    """q3s_context_set_path_stats: every row of a launch is counted once, on
    the path its parameters lead to, and the results equal a launch without
    the counters."""
    ctx = q3s.Context(0)
    R = 2048
    w = workloads.bandwidth(DEV, rows=R, top_k=50)
    params = np.repeat(q3s.make_params(1, top_k=50), R)
    params["do_sample"][:256] = 0                       # greedy
    params["temperature"][256:320] = -1.0               # invalid temperature
    params["top_k"][320:512] = 0                        # k off, top-p 1: general path
    params["top_k"][512:768] = 0                        # k off, top-p 0.8, sharp: nucleus
    params["top_p"][512:768] = 0.8
    params["temperature"][512:768] = 0.25
    params["top_p"][768:1024] = 0.9                     # top-k then top-p
    w.params = params
    a = w.device_args(DEV)
    p, s, u = a.pop("params"), a.pop("seeds"), a.pop("subseqs")
    t0, st0 = q3s.sample_batch(w.logits, p, s, u, ctx=ctx)
    stats = torch.zeros(2 * len(q3s.PATH_NAMES), dtype=torch.int64, device=DEV)
    ctx.set_path_stats(stats)
    t1, st1 = q3s.sample_batch(w.logits, p, s, u, ctx=ctx)
    torch.cuda.synchronize()
    ctx.set_path_stats(None)
    rep = q3s.path_report(stats)
    assert {k: v["rows"] for k, v in rep.items()} == {
        "greedy": 256, "invalid": 64, "general_rules": 192, "nucleus": 256, "topk_topp": 256,
        "topk": R - 1024}
    assert all(v["cycles_per_row"] > 0 for v in rep.values())
    assert torch.equal(t0, t1) and torch.equal(st0, st1)
    ref = oracle_tokens(w)
    np.testing.assert_array_equal(st1.cpu().numpy(), ref["status"])
    np.testing.assert_array_equal(t1.cpu().numpy().view(np.uint32), ref["tokens"])
