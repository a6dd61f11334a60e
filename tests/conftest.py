"""Shared pytest setup: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device and the built sampler library; every
other test runs on CPU.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "oracle", ROOT / "qwen3tts-rs_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle  # noqa: WPS433 - test infrastructure
    oracle.lib()
    return oracle
