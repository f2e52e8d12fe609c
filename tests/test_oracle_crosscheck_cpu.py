"""Cross-check of the numpy oracle's RoFormer forward (oracle/roformer.py) against an independent
float64 PyTorch re-expression (tests/_torch_roformer.py: unfolded norms, SDPA attention,
complex-number RoPE, erf GELU, index_add_ scatter). The reference ships no golden RoFormer output,
so this guards the oracle against a misreading of network.rs / roformer.rs that a single
restatement would carry into every parity test of the CUDA path.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from ancha_b200 import synthetic  # noqa: E402
from ancha_b200.config import ModelConfig  # noqa: E402
from oracle import roformer as oracle_model  # noqa: E402
from tests._torch_roformer import TorchRoformer  # noqa: E402


def _compare(package, frames, seed):
    rng = np.random.default_rng(seed)
    spectrum = rng.standard_normal((frames, 1025 * 4)) * 0.5
    a = oracle_model.Roformer(package).forward(spectrum)
    b = TorchRoformer(package).forward(torch.from_numpy(spectrum)).numpy()
    assert a.shape == b.shape
    scale = np.abs(a).max()
    err = np.abs(a - b).max()
    print(f"oracle vs torch float64: max |d| {err:.3e} (scale {scale:.3e})")
    assert err <= 1e-10 * max(scale, 1.0)


@pytest.mark.parametrize("family", ["mel-band-roformer", "bs-roformer"])
@pytest.mark.parametrize("kind", ["tiny", "kernel"])
def test_fixture_packages(tmp_path, family, kind):
    d = str(tmp_path / "pkg")
    (synthetic.tiny_package if kind == "tiny" else synthetic.kernel_package)(d, family)
    _compare(d, 37, 1)


def test_benchmark_mel_network(mel_seeded_package):
    """The seeded Mel-Band RoFormer of BASELINE config 1 on a few frames."""
    _compare(mel_seeded_package, 9, 2)


def test_benchmark_bs_network(tmp_path):
    """The seeded BS-RoFormer 512 of BASELINE config 3 on a few frames."""
    d = str(tmp_path / "pkg")
    synthetic.seeded_package(d, ModelConfig.bs_roformer_512())
    _compare(d, 5, 2)
