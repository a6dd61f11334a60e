#!/usr/bin/env python3
"""Regenerate the golden vectors under tests/golden/ from the reference.

Run where a checkout of the reference (qwen3tts-rs 0.2.0) is available; its
path is a required argument (nothing else needs the reference):

    python tests/golden/make_golden.py --reference <path to the checkout>

It reads the reference's own sampling fixtures
(fixtures/alignment/p02_*.json), transcribes the literal cases of its Rust unit
tests (src/talker/sampling.rs:789-1147, tests/suppression_eos_test.rs,
tests/sampling_config_test.rs) and imports its independent Python oracle
(tools/generate_deterministic_token_sequences.py) to produce extra seeded
cases.  Everything is written as compact JSON with float32 values as hex bit
patterns, so the tests never need the reference itself.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import random
import struct
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", float(x)))[0]


def hexbits(x: float) -> str:
    return "0x%08x" % struct.unpack("<I", struct.pack("<f", f32(x)))[0]


def encode_row(values: list[float]) -> dict:
    """Compact row: the most common value plus the exceptions, as f32 bits."""
    bits = [hexbits(v) for v in values]
    counts: dict[str, int] = {}
    for b in bits:
        counts[b] = counts.get(b, 0) + 1
    fill = max(counts, key=lambda b: counts[b])
    return {"n": len(bits), "fill": fill, "at": [[i, b] for i, b in enumerate(bits) if b != fill]}


def load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    assert spec.loader is not None
    spec.loader.exec_module(mod)
    return mod


def philox_vectors(ref: Path) -> dict:
    src = json.loads((ref / "fixtures/alignment/p02_philox_vectors.json").read_text())
    cases = []
    for c in src["cases"]:
        cases.append({
            "name": c["name"],
            "seed": c["seed"],
            "ctr_lo": c["ctr_lo"],
            "samples": [{"subsequence": s["subsequence"], "words": s["words"],
                         "uniform_bits": s["uniform_bits"]} for s in c["samples"]],
        })
    # sampling.rs:931-985: known words of the zero key.
    cases.append({
        "name": "sampling_rs_zero_key_words",
        "seed": "0",
        "ctr_lo": 0,
        "samples": [{"subsequence": "0",
                     "words": [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8],
                     "uniform_bits": "0x3ecc4fd2"}],
    })
    return {"source": "fixtures/alignment/p02_philox_vectors.json; src/talker/sampling.rs:931-985",
            "cases": cases}


def repetition_vectors(ref: Path) -> dict:
    src = json.loads((ref / "fixtures/alignment/p02_repetition_penalty_vectors.json").read_text())
    keep = ("name", "logit_bits", "history", "suppress_from", "allow_suppressed_token", "options",
            "after_repetition_bits", "candidates_after_repetition", "after_temperature_bits",
            "candidates_after_temperature", "seed")
    cases = []
    for c in src["cases"]:
        d = {k: c[k] for k in keep}
        d["candidates_before_repetition"] = [x["idx"] for x in c["candidates_before_repetition"]]
        d["candidates_before_repetition_bits"] = [x["logit_bits"] for x in c["candidates_before_repetition"]]
        d["samples"] = [{"expected": s["expected"], "uniform_bits": s["uniform_bits"]}
                        for s in c["samples"]]
        cases.append(d)
    return {"source": "fixtures/alignment/p02_repetition_penalty_vectors.json", "cases": cases}


def sequence_vectors(ref: Path) -> dict:
    src = json.loads((ref / "fixtures/alignment/p02_deterministic_token_sequences.json").read_text())
    cases = []
    for c in src["cases"]:
        calls = []
        for call in c["calls"]:
            calls.append({
                "frame": call["frame"],
                "codebook": call["codebook"],
                "logits": encode_row(call["logits"]),
                "options": call["options"],
                "history": call["history"],
                "suppress_from": call["suppress_from"],
                "allow_token": call["allow_token"],
                "expected": call["expected"],
                "subsequence": call["subsequence"],
            })
        cases.append({"id": c["id"], "seed": c["seed"], "frames": c["frames"],
                      "c0_history": c["c0_history"], "draw_count": c["draw_count"],
                      "calls": calls})
    return {"source": "fixtures/alignment/p02_deterministic_token_sequences.json", "cases": cases}


def suppression_vectors(ref: Path) -> dict:
    src = json.loads((ref / "fixtures/alignment/p02_suppression_eos_vectors.json").read_text())
    cases = []
    for c in src["cases"]:
        allowed = sorted(c["allowed"])
        # Compress as ranges [lo, hi).
        ranges = []
        for a in allowed:
            if ranges and ranges[-1][1] == a:
                ranges[-1][1] = a + 1
            else:
                ranges.append([a, a + 1])
        cases.append({"vocab_size": c["vocab_size"], "suppress_from": c["suppress_from"],
                      "eos": c["eos"], "step": c["step"], "allowed_ranges": ranges})
    return {"source": "fixtures/alignment/p02_suppression_eos_vectors.json", "cases": cases}


def config_vectors(ref: Path) -> dict:
    src = json.loads((ref / "fixtures/alignment/p02_sampling_config_matrix.json").read_text())
    models = []
    for m in src["models"]:
        models.append({"model_id": m["model_id"],
                       "raw": m["generation_config"]["raw"],
                       "resolved": m["generation_config"]["resolved"]})
    return {"source": "fixtures/alignment/p02_sampling_config_matrix.json",
            "cases": src["cases"], "models": models}


INF = float("inf")
NAN = float("nan")


def unit_literals() -> dict:
    """Literal cases of the reference's Rust unit tests, transcribed as data.

    kind "logits": sample_logits(logits, options, suppress_from, allow,
    history, || r) == expected (the helper drives sample_logits_with_scratch
    directly with a fixed draw).  kind "greedy_select": greedy_select(...).
    """
    g = {"temperature": 0.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0}
    sup = [0.0] * 2050
    sup[2], sup[2048], sup[2049] = 1.0, 10.0, 9.0
    eight = [0.0] * 8
    eight[3], eight[7] = 10.0, 20.0
    eos8 = [0.0] * 8
    eos8[7] = 20.0
    cases = [
        ("sampling.rs:790 greedy_returns_highest_finite_logit", [0.0, 3.0, -INF, 2.0], g, None, None, [], 0.5, 1),
        ("sampling.rs:803 greedy_skips_repetition_penalty", [1.0, 0.9],
         {"temperature": 0.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 2.0}, None, None, [0], 0.5, 0),
        ("sampling.rs:821 suppression_blocks_control_tokens_but_allows_eos", sup, g, 2048, 2049, [], 0.0, 2049),
        ("sampling.rs:839 top_k_sampling_limits_candidates", [10.0, 9.0, 8.0],
         {"temperature": 1.0, "top_k": 1, "top_p": 1.0, "repetition_penalty": 1.0}, None, None, [], 0.99, 0),
        ("sampling.rs:857 top_k_keeps_all_kth_score_ties_in_vocab_order", [4.0, 3.0, 3.0, -10.0],
         {"temperature": 1.0, "top_k": 2, "top_p": 1.0, "repetition_penalty": 1.0}, None, None, [], 0.99, 2),
        ("sampling.rs:1095 run_reference_sampler_reorders_temperature_before_top_k", [1.0, 2.0, 3.0, -INF],
         {"temperature": 0.5, "top_k": 1, "top_p": 1.0, "repetition_penalty": 1.0}, 4, None, [], 0.999, 2),
        ("suppression_eos_test.rs:77 sampled_literal_vectors (masked)", eight,
         {"temperature": 1.0, "top_k": 1, "top_p": 1.0, "repetition_penalty": 1.0}, 4, None, [], None, 3),
        ("suppression_eos_test.rs:77 sampled_literal_vectors (eos allowed)", eos8,
         {"temperature": 1.0, "top_k": 1, "top_p": 1.0, "repetition_penalty": 1.0}, 4, 7, [], None, 7),
    ]
    out = []
    for name, logits, opts, sf, allow, hist, r, expected in cases:
        out.append({"name": name, "kind": "logits", "logits": encode_row(logits), "options": opts,
                    "suppress_from": sf, "allow_token": allow, "history": hist,
                    "uniform": r, "expected": expected})
    out.append({"name": "suppression_eos_test.rs:132 code_predictor_reserved_tokens_are_not_suppressed",
                "kind": "greedy_select", "logits": encode_row([0.0, 10.0]), "suppress_from": None,
                "allow_token": None, "expected": 1})
    # sampling.rs:1108-1147 penalty bit patterns.
    pen = {"name": "sampling.rs:1108 apply_repetition_penalty_produces_expected_bits",
           "logits": [hexbits(v) for v in [1.0, -2.0, 0.0, -0.0, 7.5]],
           "history": [0, 3, 1, 3, 1, 99], "penalty": 1.5,
           "expected": [hexbits(f32(1.0) / f32(1.5)), hexbits(-3.0), hexbits(0.0), "0x80000000",
                        hexbits(7.5)]}
    # Failure cases: no Philox consumed (sampling.rs:1056-1092; suppression_eos_test.rs:108-129)
    # and rejected options (sampling.rs:1028-1053; repetition_penalty_test.rs:329-363).
    failures = [
        {"name": "sampling.rs:1056 all suppressed", "logits": encode_row([0.0, 1.0, -1.0]),
         "options": {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0},
         "do_sample": True, "suppress_from": 0, "allow_token": None, "seed": 42},
        {"name": "sampling.rs:1073 all non-finite", "logits": encode_row([NAN, INF, -INF]),
         "options": {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0},
         "do_sample": True, "suppress_from": None, "allow_token": None, "seed": 1337},
        {"name": "suppression_eos_test.rs:108 suppressed", "logits": encode_row([0.0, 1.0]),
         "options": {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0},
         "do_sample": True, "suppress_from": 0, "allow_token": None, "seed": 1},
        {"name": "suppression_eos_test.rs:120 non-finite suppressed", "logits": encode_row([NAN, -INF]),
         "options": {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0},
         "do_sample": True, "suppress_from": 0, "allow_token": None, "seed": 1},
    ]
    for t in [0.0, -1.0, NAN, INF]:
        failures.append({"name": "sampling.rs:1031 temperature %r" % t, "logits": encode_row([0.0, 1.0]),
                         "options": {"temperature": t, "top_k": 0, "top_p": 1.0, "repetition_penalty": 1.0},
                         "do_sample": True, "suppress_from": None, "allow_token": None, "seed": 0})
    for p in [0.0, -1.0, 1.1, NAN, INF]:
        failures.append({"name": "sampling.rs:1042 top_p %r" % p, "logits": encode_row([0.0, 1.0]),
                         "options": {"temperature": 1.0, "top_k": 0, "top_p": p, "repetition_penalty": 1.0},
                         "do_sample": True, "suppress_from": None, "allow_token": None, "seed": 0})
    for rp in [0.0, -1.5, NAN]:
        failures.append({"name": "repetition_penalty_test.rs:329 penalty %r" % rp,
                         "logits": encode_row([0.0, 1.0]),
                         "options": {"temperature": 1.0, "top_k": 0, "top_p": 1.0, "repetition_penalty": rp},
                         "do_sample": True, "suppress_from": None, "allow_token": None, "seed": 1})
    return {"source": "src/talker/sampling.rs:789-1147; tests/suppression_eos_test.rs; "
                      "tests/repetition_penalty_test.rs",
            "cases": out, "penalty_bits": pen, "failures": failures}


def python_oracle_vectors(ref: Path, count: int = 300) -> dict:
    """Seeded extra cases decided by the reference's own Python oracle
    (tools/generate_deterministic_token_sequences.py: oracle()).

    That oracle divides by the temperature and evaluates exp and the top-p
    probabilities in binary64, while the Rust sampler multiplies by an f32
    reciprocal.  The two agree bit for bit when the temperature is a power of
    two, every logit difference is exact in f32 (multiples of 1/128 below 16),
    the penalty is a power of two, and top_p is 1, so cases are drawn there.
    """
    mod = load_module(ref / "tools/generate_deterministic_token_sequences.py", "ref_det_oracle")
    rng = random.Random(20240531)
    cases = []
    for case_id in range(count):
        n = rng.choice([2, 3, 5, 8, 17, 31, 64, 100, 128, 257])
        logits = [rng.randint(-600, 600) / 64.0 for _ in range(n)]
        for _ in range(rng.randint(0, 3)):  # exact ties
            logits[rng.randrange(n)] = logits[rng.randrange(n)]
        if rng.random() < 0.2:
            logits[rng.randrange(n)] = -INF
        if rng.random() < 0.1:
            logits[rng.randrange(n)] = NAN
        do_sample = rng.random() < 0.8
        temperature = rng.choice([0.5, 1.0, 2.0])
        top_k = rng.choice([0, 0, 1, 2, 3, 5, 10, n, n + 3])
        rp = rng.choice([1.0, 2.0, 0.5, 4.0]) if do_sample else 1.0
        history = [rng.randrange(n + 4) for _ in range(rng.randint(0, 8))]
        sf, allow = None, None
        if rng.random() < 0.3 and n > 2:
            sf = rng.randrange(1, n)
            allow = rng.choice([None, rng.randrange(n)])
        seed = rng.randrange(1 << 64)
        subseq = rng.choice([0, 1, 7, rng.randrange(1 << 64)])
        opts = {"do_sample": do_sample, "temperature": temperature, "top_k": top_k, "top_p": 1.0,
                "repetition_penalty": rp}
        try:
            token, drew = mod.oracle(logits, opts, history, suppress_from=sf, allow=allow,
                                     seed=seed, subseq=subseq)
            status = "ok"
        except ValueError:
            token, drew, status = None, False, "no_candidate"
        # Logits are multiples of 1/64: store the integer numerators.
        q64 = [("nan" if v != v else "-inf" if v == -INF else int(v * 64)) for v in logits]
        cases.append({"id": case_id, "logits_q64": q64, "options": opts,
                      "history": history, "suppress_from": sf, "allow_token": allow,
                      "seed": str(seed), "subsequence": str(subseq),
                      "expected": token, "drew": bool(drew), "status": status})
    return {"source": "tools/generate_deterministic_token_sequences.py oracle() on seeded cases",
            "cases": cases}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True,
                    help="path of the reference checkout (qwen3tts-rs 0.2.0)")
    args = ap.parse_args()
    ref = args.reference
    if not (ref / "src/talker/sampling.rs").exists():
        print("reference checkout not found at %s" % ref, file=sys.stderr)
        return 2
    outputs = {
        "philox.json": philox_vectors(ref),
        "repetition_penalty.json": repetition_vectors(ref),
        "token_sequences.json": sequence_vectors(ref),
        "suppression_eos.json": suppression_vectors(ref),
        "sampling_config.json": config_vectors(ref),
        "unit_literals.json": unit_literals(),
        "python_oracle_cases.json": python_oracle_vectors(ref),
    }
    for name, payload in outputs.items():
        text = json.dumps(payload, separators=(",", ":"), sort_keys=True,
                          allow_nan=True) + "\n"
        (HERE / name).write_text(text)
        print("wrote %s (%d bytes)" % (name, len(text)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
