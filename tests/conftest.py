"""Shared fixtures. Tests marked ``gpu`` need a B200 and the built
libitts_cfm.so; everything else runs on CPU."""
from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "index-tts2-metal_b200"
for p in (str(PKG), str(REPO / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import mit2  # noqa: E402

BUNDLE_ROOT = Path(os.environ.get("ITTS_TEST_BUNDLES", Path(tempfile.gettempdir()) / "itts_cfm_test_bundles"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def bundle_path(seed: int, init: str) -> Path:
    return mit2.make_dit_bundle(BUNDLE_ROOT / f"seed{seed}_{init}", seed=seed, init=init)


@pytest.fixture(scope="session")
def unit_bundle() -> Path:
    return bundle_path(0, "unit")


@pytest.fixture(scope="session")
def baseline_bundle() -> Path:
    return bundle_path(0, "baseline")


@pytest.fixture(scope="session")
def unit_tensors(unit_bundle):
    return mit2.bundle_f32(unit_bundle)


@pytest.fixture(scope="session")
def port_unit(unit_tensors):
    import oracle

    return oracle.PortOracle(unit_tensors)


@pytest.fixture(scope="session")
def baseline_tensors(baseline_bundle):
    return mit2.bundle_f32(baseline_bundle)


@pytest.fixture(scope="session")
def port_baseline(baseline_tensors):
    import oracle

    return oracle.PortOracle(baseline_tensors)


@pytest.fixture(scope="session")
def vocoder_bundle() -> Path:
    return mit2.make_vocoder_bundle(BUNDLE_ROOT / "bigvgan_seed0", seed=0)


@pytest.fixture(scope="session")
def vocoder_tensors(vocoder_bundle):
    return mit2.bundle_f32(vocoder_bundle)


@pytest.fixture(scope="session")
def port_vocoder(vocoder_tensors):
    import oracle

    return oracle.VocoderOracle(vocoder_tensors)


@pytest.fixture(scope="session")
def condition_bundle() -> Path:
    return mit2.make_condition_bundle(BUNDLE_ROOT / "length_regulator_seed0", seed=0)


@pytest.fixture(scope="session")
def port_condition(condition_bundle):
    import oracle

    return oracle.ConditionOracle(mit2.bundle_f32(condition_bundle))


@pytest.fixture(scope="session")
def gpt_bundle() -> Path:
    return mit2.make_gpt_bundle(BUNDLE_ROOT / "gpt_seed0", seed=0)


@pytest.fixture(scope="session")
def gpt_oracle(gpt_bundle):
    import gpt_oracle as G

    return G.GptOracle(mit2.bundle_f32(gpt_bundle))


def _gpu_ctx(bundle):
    import itts_cfm

    return itts_cfm.Context(bundle, device=0)


@pytest.fixture(scope="session")
def ctx_unit(unit_bundle):
    c = _gpu_ctx(unit_bundle)
    yield c
    c.close()


@pytest.fixture(scope="session")
def ctx_baseline(baseline_bundle):
    c = _gpu_ctx(baseline_bundle)
    yield c
    c.close()


@pytest.fixture
def rng():
    return np.random.default_rng(1234)
