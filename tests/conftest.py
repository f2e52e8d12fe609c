"""Shared pytest setup: the ``gpu`` marker and the repository root on ``sys.path``."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) and the built CUDA library")


import pytest  # noqa: E402


@pytest.fixture(scope="session")
def mel_seeded_package(tmp_path_factory):
    """The benchmark's seeded Mel-Band RoFormer package (dim 384, depth 6, N(0, 0.02) weights),
    written once per session: its 180 M mask-head weights take a while to draw and hash."""
    from ancha_b200 import synthetic
    from ancha_b200.config import ModelConfig
    d = str(tmp_path_factory.mktemp("mel_seeded") / "pkg")
    synthetic.seeded_package(d, ModelConfig.mel_karaoke())
    return d
