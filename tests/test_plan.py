"""Sampling plan on CPU: generation_config parsing, the public overrides and
the per-branch row parameters, against the reference's config matrix fixture
(fixtures/alignment/p02_sampling_config_matrix.json, via tests/golden/) and
the literal cases of tests/sampling_config_test.rs:255-266."""
import json
import math
from pathlib import Path

import pytest

import q3s
from q3s import plan

GOLDEN = Path(__file__).resolve().parent / "golden" / "sampling_config.json"


def _opts(d):
    return q3s.SamplingOptions(d["temperature"], d["top_k"], d["top_p"], d["repetition_penalty"])


def _cases():
    return json.loads(GOLDEN.read_text())["cases"]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_config_matrix_case(case, tmp_path):
    path = tmp_path / "generation_config.json"
    path.write_text(json.dumps(case["generation_config"], indent=2))
    if case.get("expect_error"):
        with pytest.raises(plan.ConfigError):
            plan.GenerationSamplingConfig.from_path(path)
        return
    cfg = plan.GenerationSamplingConfig.from_path(path)
    exp = case["expected"]
    assert cfg.talker.do_sample == exp["talker"]["do_sample"]
    assert cfg.subtalker.do_sample == exp["subtalker"]["do_sample"]
    so = case["synthesis_options"]
    p = plan.resolve_effective_sampling_plan(cfg, so["temperature"], so["top_k"], so["top_p"])
    assert plan.route(p) == exp["route"]
    assert p.talker.options == _opts(exp["talker"]["options"])
    assert p.subtalker.options == _opts(exp["subtalker"]["options"])


def test_model_generation_configs_resolve():
    for m in json.loads(GOLDEN.read_text())["models"]:
        cfg = plan.GenerationSamplingConfig.from_parsed(m["raw"])
        r = m["resolved"]
        assert cfg.talker.do_sample == r["talker"]["do_sample"], m["model_id"]
        assert cfg.subtalker.do_sample == r["subtalker"]["do_sample"], m["model_id"]
        assert cfg.talker.options == _opts(r["talker"]["options"]), m["model_id"]
        assert cfg.subtalker.options == _opts(r["subtalker"]["options"]), m["model_id"]


def test_missing_file_means_defaults(tmp_path):
    assert plan.GenerationSamplingConfig.from_model_dir(tmp_path) == \
        plan.GenerationSamplingConfig.default()
    (tmp_path / "generation_config.json").write_text("{not json")
    with pytest.raises(plan.ConfigError, match="invalid generation_config.json"):
        plan.GenerationSamplingConfig.from_model_dir(tmp_path)


def test_public_overrides_are_validated():
    cfg = plan.GenerationSamplingConfig.default()
    for t in (math.nan, math.inf, -math.inf):
        with pytest.raises(plan.ConfigError, match="temperature must be finite"):
            plan.resolve_effective_sampling_plan(cfg, t, 50, 1.0)
    for p in (0.0, -0.1, 1.1, math.nan, math.inf):
        with pytest.raises(plan.ConfigError, match="top_p"):
            plan.resolve_effective_sampling_plan(cfg, 0.9, 50, p)
    greedy = plan.resolve_effective_sampling_plan(cfg, 0.0, 0, 1.0)
    assert not greedy.talker.do_sample and greedy.subtalker.do_sample


def test_row_params_follow_the_caller_contract():
    p = plan.resolve_effective_sampling_plan(plan.GenerationSamplingConfig.default(), 0.9, 50, 1.0)
    for step, allow in ((0, q3s.NONE), (1, q3s.NONE), (2, 2150), (40, 2150)):
        r = plan.talker_row_params(p, step)
        assert int(r["suppress_from"][0]) == 2048 and int(r["allow_token"][0]) == allow
        assert int(r["do_sample"][0]) == 1
        assert plan.row_options(r) == q3s.SamplingOptions(0.9, 50, 1.0, 1.05)
    c = plan.subtalker_row_params(p)
    assert int(c["suppress_from"][0]) == q3s.NONE and float(c["repetition_penalty"][0]) == 1.0
    g = plan.resolve_effective_sampling_plan(
        plan.GenerationSamplingConfig.from_parsed({"subtalker_dosample": False}), 0.9, 50, 1.0)
    cg = plan.subtalker_row_params(g)
    assert float(cg["temperature"][0]) == -1.0 and int(cg["do_sample"][0]) == 0
    with pytest.raises(ValueError, match="reserved"):
        plan.talker_row_params(p, 0, vocab=512)
    with pytest.raises(ValueError, match="EOS"):
        plan.talker_row_params(p, 0, vocab=3072, eos=100)
