"""Sampling plan: generation_config.json and the public synthesis options to
the per-branch SamplingOptions the sampler is called with, and the
q3s_row_params of a talker (codebook 0) row and a code-predictor
(codebooks 1..15) row.

Follows src/text_frontend/model_catalog.rs:23-58 (defaults), :91-118
(resolve_effective_sampling_plan), :123-215 (default, from_path,
from_model_dir, from_parsed) and :234-263 (validation); the row rules follow src/talker/talker.rs:452-461, 511-519
(suppression of the 1024 reserved ids, EOS allowed from step 2) and
src/talker/code_predictor.rs:357-364 (greedy as temperature -1, no
suppression, no history, repetition penalty 1).
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, replace
from pathlib import Path

import numpy as np

from . import NONE, SamplingOptions, make_params

GENERATION_CONFIG_FILE = "generation_config.json"
RESERVED_TALKER_IDS = 1024


class ConfigError(ValueError):
    """crate::Error::Config of the reference (same message texts)."""


@dataclass(frozen=True)
class BranchSamplingConfig:
    do_sample: bool
    options: SamplingOptions


@dataclass(frozen=True)
class GenerationSamplingConfig:
    talker: BranchSamplingConfig
    subtalker: BranchSamplingConfig

    @staticmethod
    def default() -> "GenerationSamplingConfig":
        return GenerationSamplingConfig(
            BranchSamplingConfig(True, SamplingOptions(0.9, 50, 1.0, 1.05)),
            BranchSamplingConfig(True, SamplingOptions(0.9, 50, 1.0, 1.0)))

    @staticmethod
    def from_parsed(cfg: dict) -> "GenerationSamplingConfig":
        """Fields absent from `cfg` take the defaults; the subtalker's
        repetition penalty is always 1.0."""
        d = GenerationSamplingConfig.default()

        def get(key, default):
            v = cfg.get(key)
            return default if v is None else v
        talker = SamplingOptions(float(get("temperature", d.talker.options.temperature)),
                                 int(get("top_k", d.talker.options.top_k)),
                                 float(get("top_p", d.talker.options.top_p)),
                                 float(get("repetition_penalty",
                                           d.talker.options.repetition_penalty)))
        sub = SamplingOptions(float(get("subtalker_temperature", d.subtalker.options.temperature)),
                              int(get("subtalker_top_k", d.subtalker.options.top_k)),
                              float(get("subtalker_top_p", d.subtalker.options.top_p)), 1.0)
        do_sample = bool(get("do_sample", d.talker.do_sample))
        sub_do_sample = bool(get("subtalker_dosample", d.subtalker.do_sample))
        validate_generation_sampling("talker", do_sample, talker)
        validate_generation_sampling("subtalker", sub_do_sample, sub)
        return GenerationSamplingConfig(BranchSamplingConfig(do_sample, talker),
                                        BranchSamplingConfig(sub_do_sample, sub))

    @staticmethod
    def from_path(path) -> "GenerationSamplingConfig":
        p = Path(path)
        try:
            payload = p.read_text()
        except OSError as err:
            raise ConfigError(f"unable to read generation_config.json at {p}: {err}") from None
        try:
            parsed = json.loads(payload)
            if not isinstance(parsed, dict):
                raise ValueError("expected a JSON object")
        except ValueError as err:
            raise ConfigError(f"invalid generation_config.json at {p}: {err}") from None
        return GenerationSamplingConfig.from_parsed(parsed)

    @staticmethod
    def from_model_dir(model_dir) -> "GenerationSamplingConfig":
        """A missing generation_config.json means the defaults."""
        p = Path(model_dir) / GENERATION_CONFIG_FILE
        if not p.exists():
            return GenerationSamplingConfig.default()
        return GenerationSamplingConfig.from_path(p)


def validate_generation_sampling(branch: str, do_sample: bool, s: SamplingOptions) -> None:
    if not math.isfinite(s.top_p) or s.top_p <= 0.0 or s.top_p > 1.0:
        raise ConfigError(f"generation_config[{branch}].top_p must be finite and in (0.0, 1.0]")
    if not math.isfinite(s.repetition_penalty) or s.repetition_penalty <= 0.0:
        raise ConfigError(
            f"generation_config[{branch}].repetition_penalty must be finite and > 0.0")
    if not math.isfinite(s.temperature):
        raise ConfigError(f"generation_config[{branch}].temperature must be finite")
    if do_sample and s.temperature <= 0.0:
        raise ConfigError(
            f"generation_config[{branch}].temperature must be > 0.0 when do_sample=true")


@dataclass(frozen=True)
class EffectiveSamplingPlan:
    talker: BranchSamplingConfig
    subtalker: BranchSamplingConfig

    def uses_explicit_sampler(self) -> bool:
        return self.talker.do_sample or self.subtalker.do_sample


def resolve_effective_sampling_plan(config: GenerationSamplingConfig, temperature: float,
                                    top_k: int, top_p: float) -> EffectiveSamplingPlan:
    """The public overrides replace the talker's temperature, top_k and top_p;
    the talker samples only when its config says so and temperature > 0."""
    if not math.isfinite(temperature):
        raise ConfigError("SynthesisOptions.temperature must be finite")
    if not math.isfinite(top_p) or top_p <= 0.0 or top_p > 1.0:
        raise ConfigError("SynthesisOptions.top_p must be finite and in (0.0, 1.0]")
    talker = replace(config.talker.options, temperature=float(temperature),
                     top_k=int(top_k) & 0xFFFFFFFF, top_p=float(top_p))
    return EffectiveSamplingPlan(
        BranchSamplingConfig(config.talker.do_sample and temperature > 0.0, talker),
        config.subtalker)


def talker_row_params(plan: EffectiveSamplingPlan, step: int, vocab: int = 3072,
                      eos: int = 2150) -> np.ndarray:
    """q3s_row_params of a codebook-0 row at generation step `step`: the last
    1024 ids suppressed, EOS allowed from step 2 on."""
    suppress_from = vocab - RESERVED_TALKER_IDS
    if suppress_from < 0:
        raise ValueError("Talker vocabulary must contain at least 1024 reserved tokens")
    if eos >= vocab or eos < suppress_from:
        raise ValueError("Talker codec EOS must be inside reserved vocabulary suffix")
    o = plan.talker.options
    return make_params(1, temperature=o.temperature, top_k=o.top_k, top_p=o.top_p,
                       repetition_penalty=o.repetition_penalty,
                       do_sample=1 if plan.talker.do_sample else 0,
                       suppress_from=suppress_from, allow_token=eos if step >= 2 else NONE)


def subtalker_row_params(plan: EffectiveSamplingPlan) -> np.ndarray:
    """q3s_row_params of a code-predictor row (codebooks 1..15): no
    suppression, no history; a greedy branch is temperature -1."""
    o = plan.subtalker.options
    t = o.temperature if plan.subtalker.do_sample else -1.0
    return make_params(1, temperature=t, top_k=o.top_k, top_p=o.top_p,
                       repetition_penalty=o.repetition_penalty, do_sample=1 if t > 0.0 else 0,
                       suppress_from=NONE, allow_token=NONE)


def row_options(params: np.ndarray, index: int = 0) -> SamplingOptions:
    p = params[index]
    return SamplingOptions(float(p["temperature"]), int(p["top_k"]), float(p["top_p"]),
                           float(p["repetition_penalty"]))


def route(plan: EffectiveSamplingPlan) -> str:
    """The generation entry the reference takes for a plan."""
    return "generate_sampled" if plan.uses_explicit_sampler() else "generate"


__all__ = ["BranchSamplingConfig", "ConfigError", "EffectiveSamplingPlan",
           "GenerationSamplingConfig", "resolve_effective_sampling_plan", "route",
           "row_options", "subtalker_row_params", "talker_row_params",
           "validate_generation_sampling"]
