"""Device-resident decode frame: q3s_commit_rows after each of a frame's 16
batched launches (1 talker row + 15 code-predictor groups per stream) keeps
the ids, the Philox counters and the c0 history on the device, and the frame
is read back once at its end.  Checked against per-stream replays of the
reference's call order with the oracle (one Sampler per stream, as
talker.rs:500-566 and code_predictor.rs:337-427 drive it on the host: the
c0 call with the accumulated history, then 15 calls with none, the frame
ending at the first error).

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
import embed_oracle  # noqa: E402

DEV = torch.device("cuda:0")
GROUPS = 16


def opts(p) -> dict:
    return {"temperature": float(p["temperature"]), "top_k": int(p["top_k"]),
            "top_p": float(p["top_p"]), "repetition_penalty": float(p["repetition_penalty"])}


def test_four_mode_cross_product_on_device():
    """tests/sampling_config_test.rs:199-226 of the reference: seed 7, one c0
    call with history [0] and 15 calls without, in the four (talker,
    sub-talker) do_sample modes; the counter ends at talker + 15 * sub-talker.
    Here the 16 calls of the four streams are 16 launches, each followed by
    the device-side commit, with no host read until the end."""
    modes = [(t, s) for t in (False, True) for s in (False, True)]
    S = len(modes)
    x = torch.tensor([[0.1, 0.9]] * S, dtype=torch.float32, device=DEV)
    seeds = torch.full((S,), 7, dtype=torch.int64, device=DEV)
    subseqs = torch.zeros(S, dtype=torch.int64, device=DEV)
    codes = torch.zeros((S, GROUPS), dtype=torch.int32, device=DEV)
    fstat = torch.zeros(S, dtype=torch.uint8, device=DEV)
    hist = torch.zeros(S, dtype=torch.int16, device=DEV)
    hoff = torch.arange(S + 1, dtype=torch.int64, device=DEV)
    for g in range(GROUPS):
        p = q3s.make_params(S, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.5)
        p["do_sample"] = [m[0] if g == 0 else m[1] for m in modes]
        pt = torch.from_numpy(p.view(np.uint8).copy()).to(DEV)
        kw = {"history": hist, "history_offsets": hoff} if g == 0 else {}
        t, st = q3s.sample_batch(x, pt, seeds, subseqs, **kw)
        q3s.commit_rows(t, st, params=pt, subseqs=subseqs, codes=codes, group=g,
                        frame_status=fstat)
    torch.cuda.synchronize()
    got_codes = codes.cpu().numpy()
    assert fstat.cpu().numpy().tolist() == [0] * S
    assert subseqs.cpu().numpy().tolist() == [int(t) + 15 * int(s) for t, s in modes]
    o_opts = {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.5}
    for i, (ts, ss) in enumerate(modes):
        o = oracle.OracleSampler(7)
        want = []
        for g in range(GROUPS):
            st, tok = o.sample_with_mode(np.array([0.1, 0.9], np.float32), o_opts,
                                         ts if g == 0 else ss, None, None,
                                         [0] if g == 0 else [])
            assert st == 0
            want.append(tok)
        assert got_codes[i].tolist() == want
        assert o.subsequence_counter == int(subseqs[i].item()), i


def _frame_inputs(rng, S):
    """One frame's logits and parameters: a talker row per stream (3072 f32,
    N(0, 2.5^2), talker suppression) and 15 bf16 code-predictor rows of 2048."""
    talker = (rng.standard_normal((S, 3072)) * 2.5).astype(np.float32)
    cp = (rng.standard_normal((GROUPS - 1, S, 2048)) * 3.0).astype(np.float32)
    cp_bf = torch.from_numpy(cp).to(torch.bfloat16)
    pt = q3s.make_params(S, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.05,
                         suppress_from=2048, allow_token=2150)
    pc = q3s.make_params(S, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.0)
    return talker, cp_bf, pt, pc


@pytest.mark.parametrize("fused", [False, True], ids=["sample_then_commit", "sample_commit"])
def test_frames_with_failures_history_and_embedding(fused):
    """Two frames of 64 streams through the device-side commit: the c0 ids
    join each stream's fixed-capacity history on the device and penalise the
    next frame's talker call; a stream whose code-predictor logits are all
    -inf at group 7 stops there (NO_CANDIDATE), one with an invalid talker
    top_p stops at group 0, and one whose history is full stops with
    HISTORY_FULL after its draw.  The frame's codes then feed the codebook
    embedding sum straight from the device buffer.  Run with two launches per
    group (q3s_sample_batch, q3s_commit_rows) and with one
    (q3s_sample_commit)."""
    rng = np.random.default_rng(11)
    S, HCAP = 64, 512
    fail_cp, fail_topp, full = 5, 9, 13
    seeds_np = rng.integers(0, 2**63, S).astype(np.uint64)
    sub0 = rng.integers(0, 1000, S).astype(np.uint64)
    lens = rng.integers(0, 300, S)
    lens[full] = HCAP
    hist_np = np.zeros(S * HCAP, np.uint16)
    for s in range(S):
        hist_np[s * HCAP: s * HCAP + lens[s]] = rng.integers(0, 2048, lens[s])
    seeds = torch.from_numpy(seeds_np.view(np.int64)).to(DEV)
    subseqs = torch.from_numpy(sub0.view(np.int64)).to(DEV)
    hist = torch.from_numpy(hist_np.view(np.int16)).to(DEV)
    hstart = torch.arange(S, dtype=torch.int64, device=DEV) * HCAP
    hend = hstart + torch.from_numpy(lens.astype(np.int64)).to(DEV)
    hlim = hstart + HCAP
    samplers = [oracle.OracleSampler(int(seeds_np[s])) for s in range(S)]
    for s in range(S):
        samplers[s].subsequence_counter = int(sub0[s])
    histories = [list(hist_np[s * HCAP: s * HCAP + lens[s]]) for s in range(S)]
    stopped = [0] * S  # status at which a stream's frames stopped (0: running)
    for frame in range(2):
        talker, cp_bf, pt, pc = _frame_inputs(rng, S)
        if frame == 0:
            cp_bf[7 - 1, fail_cp] = float("-inf")
            pt["top_p"][fail_topp] = 1.5
        codes = torch.zeros((S, GROUPS), dtype=torch.int32, device=DEV)
        fstat = torch.zeros(S, dtype=torch.uint8, device=DEV)
        for s in range(S):  # streams that stopped earlier stay stopped
            if stopped[s]:
                fstat[s] = stopped[s]
        ptd = torch.from_numpy(pt.view(np.uint8).copy()).to(DEV)
        pcd = torch.from_numpy(pc.view(np.uint8).copy()).to(DEV)
        xt = torch.from_numpy(talker).to(DEV)
        xc = cp_bf.to(DEV)
        if fused:
            q3s.sample_commit(xt, ptd, seeds, subseqs, codes=codes, group=0, frame_status=fstat,
                              commit_history=hist, history_limits=hlim, history=hist,
                              history_offsets=hstart, history_ends=hend)
            for g in range(1, GROUPS):
                q3s.sample_commit(xc[g - 1], pcd, seeds, subseqs, codes=codes, group=g,
                                  frame_status=fstat)
        else:
            t, st = q3s.sample_batch(xt, ptd, seeds, subseqs, history=hist,
                                     history_offsets=hstart, history_ends=hend)
            q3s.commit_rows(t, st, params=ptd, subseqs=subseqs, codes=codes, group=0,
                            frame_status=fstat, history=hist, history_ends=hend,
                            history_limits=hlim)
            for g in range(1, GROUPS):
                t, st = q3s.sample_batch(xc[g - 1], pcd, seeds, subseqs)
                q3s.commit_rows(t, st, params=pcd, subseqs=subseqs, codes=codes, group=g,
                                frame_status=fstat)
        # The embedding sum reads the frame's codes on the device.
        H = 256
        vocabs = [3072] + [2048] * (GROUPS - 1)
        tables = [(torch.randn((v, H), device=DEV) * 0.05).to(torch.bfloat16) for v in vocabs]
        emb, est = q3s.embed_sum(codes, tables)
        torch.cuda.synchronize()
        got_codes = codes.cpu().numpy().view(np.uint32)
        got_stat = fstat.cpu().numpy()
        got_sub = subseqs.cpu().numpy().view(np.uint64)
        got_end = (hend - hstart).cpu().numpy()
        got_hist = hist.cpu().numpy().view(np.uint16)
        for s in range(S):
            o = samplers[s]
            fail = stopped[s]
            want = []
            if not fail:
                for g in range(GROUPS):
                    if g == 0:
                        row, p, sf, allow, h = talker[s], pt[s], 2048, 2150, histories[s]
                    else:
                        row = cp_bf[g - 1, s].float().numpy()
                        p, sf, allow, h = pc[s], None, None, []
                    rs, tok = o.sample_with_mode(row, opts(p), True, sf, allow, h)
                    if rs:
                        fail = rs
                        break
                    want.append(tok)
                    if g == 0:
                        if len(histories[s]) >= HCAP:
                            fail = q3s.STATUS_HISTORY_FULL
                            break
                        histories[s].append(tok)
            stopped[s] = fail
            assert got_stat[s] == fail, (frame, s)
            assert got_codes[s, :len(want)].tolist() == want, (frame, s)
            assert int(got_sub[s]) == o.subsequence_counter, (frame, s)
            assert got_end[s] == len(histories[s]), (frame, s)
            assert got_hist[s * HCAP: s * HCAP + got_end[s]].tolist() == histories[s]
        assert stopped[fail_cp] == q3s.STATUS_NO_CANDIDATE
        assert stopped[fail_topp] == q3s.STATUS_INVALID_TOP_P
        assert stopped[full] == q3s.STATUS_HISTORY_FULL
        ok = got_stat == 0
        tables_bits = [t.view(torch.int16).cpu().numpy().view(np.uint16) for t in tables]
        ref, ref_st = embed_oracle.embed_sum(got_codes[ok], tables_bits, None, bf16=True)
        np.testing.assert_array_equal(
            emb[torch.from_numpy(ok).to(DEV)].view(torch.int16).cpu().numpy(),
            ref.view(np.int16))
        assert not ref_st.any()


def test_code_predictor_frame_replays_from_a_cuda_graph():
    """The 15 code-predictor groups of a frame (sampling launch + device-side
    commit each) captured once in a CUDA graph: a replay from the same
    counters gives the codes, counters and statuses of the eager frame."""
    S, G = 64, 15
    rng = np.random.default_rng(5)
    x = torch.from_numpy((rng.standard_normal((G, S, 2048)) * 3.0).astype(np.float32))
    x = x.to(torch.bfloat16).to(DEV)
    p = q3s.make_params(1, temperature=0.9, top_k=50, top_p=1.0, repetition_penalty=1.0)
    pd = torch.from_numpy(p.view(np.uint8).copy()).to(DEV)
    seeds = torch.from_numpy(rng.integers(0, 2**63, S).astype(np.int64)).to(DEV)
    sub0 = torch.from_numpy(rng.integers(0, 1000, S).astype(np.int64)).to(DEV)
    ctx = q3s.Context(0)

    def frame(subseqs, codes, fstat, stream):
        tok = torch.empty(S, dtype=torch.int32, device=DEV)
        st = torch.empty(S, dtype=torch.uint8, device=DEV)
        launches = [q3s.prepare_batch(x[g], pd, seeds, subseqs, ctx=ctx, out=(tok, st))
                    for g in range(G)]
        def run():
            fstat.zero_()
            for g in range(G):
                launches[g](stream.cuda_stream)
                q3s.commit_rows(tok, st, params=pd, subseqs=subseqs, codes=codes, group=g + 1,
                                frame_status=fstat, ctx=ctx, stream=stream.cuda_stream)
        return run, (tok, st, launches)

    s = torch.cuda.Stream(DEV)
    # Eager frame.
    sub_e = sub0.clone()
    codes_e = torch.zeros((S, 16), dtype=torch.int32, device=DEV)
    fstat_e = torch.zeros(S, dtype=torch.uint8, device=DEV)
    run_e, keep_e = frame(sub_e, codes_e, fstat_e, s)
    with torch.cuda.stream(s):
        run_e()
    torch.cuda.synchronize()
    # The same frame captured (after one warm run on its own buffers).
    sub_g = sub0.clone()
    codes_g = torch.zeros((S, 16), dtype=torch.int32, device=DEV)
    fstat_g = torch.zeros(S, dtype=torch.uint8, device=DEV)
    run_g, keep_g = frame(sub_g, codes_g, fstat_g, s)
    with torch.cuda.stream(s):
        run_g()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        run_g()
    sub_g.copy_(sub0)
    codes_g.zero_()
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(codes_g, codes_e)
    assert torch.equal(sub_g, sub_e)
    assert torch.equal(fstat_g, fstat_e) and int(fstat_g.sum()) == 0
    assert torch.equal(sub_e, sub0 + G)
