"""GPU parity of the whole RoFormer path against the oracle.

* The reference's hardware contracts on its fixture packages (tests/cuda_contracts.rs:52-104,
  403-461): full separations of the tiny (head_dim 4) and kernel (dim 128, 2×64 heads)
  packages, both families, f32 within 1e-5 of the CPU path.
* the Mel-Band RoFormer (dim 384, depth 6, 60 mel bands) with seeded
  N(0, 0.02) weights on Gaussian σ=0.1 stereo audio. Tolerances from the task: fp32 max-abs
  waveform error ≤ 1e-4 and SNR ≥ 80 dB; bf16 SNR ≥ 50 dB.
"""
import os

import numpy as np
import pytest

from tests._util import max_abs, snr_db

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from ancha_b200 import synthetic  # noqa: E402
from ancha_b200.config import ModelConfig  # noqa: E402
from ancha_b200.model import Roformer, SeparateOptions, separate, separate_pcm  # noqa: E402
from oracle import dsp  # noqa: E402
from oracle import roformer as oracle_model  # noqa: E402
from oracle import runtime as oracle_runtime  # noqa: E402


@pytest.fixture(scope="session")
def mel_package(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("mel") / "pkg")
    synthetic.seeded_package(d, ModelConfig.mel_karaoke())
    return d


@pytest.fixture(scope="session")
def mel_oracle(mel_package):
    return oracle_model.Roformer(mel_package)


def mono(n, step):
    s = (np.sin(np.arange(n, dtype=np.float32) * np.float32(step)) * np.float32(0.3)).astype(np.float32)
    return np.stack([s, s])


@pytest.mark.parametrize("family", ["bs-roformer", "mel-band-roformer"])
@pytest.mark.parametrize("kind", ["tiny", "kernel"])
def test_fixture_packages_match_oracle(tmp_path, family, kind):
    pkg = str(tmp_path / "pkg")
    (synthetic.tiny_package if kind == "tiny" else synthetic.kernel_package)(pkg, family)
    planes = mono(5003 if kind == "tiny" else 9001, 0.017 if kind == "tiny" else 0.013)
    ref, _ = oracle_runtime.separate(oracle_model.Roformer(pkg), planes)
    model = Roformer(pkg, 0, "f32")
    got, _ = separate_pcm([model], planes)
    assert got.shape == ref.shape
    assert max_abs(got, ref) < 1e-5, (family, kind, max_abs(got, ref))
    # Batching chunks changes nothing but the schedule.
    got1, _ = separate_pcm([model], planes, batch_chunks=1)
    assert max_abs(got1, got) < 1e-6


def packed_spectrum(planes):
    st = dsp.Stft(2048, 441)
    return oracle_runtime.pack_spectrum([st.forward(p) for p in planes])


@pytest.mark.parametrize("precision,tol_db", [("f32", 80.0), ("bf16", 50.0)])
def test_mel_model_masks_one_second(mel_package, mel_oracle, precision, tol_db):
    rng = np.random.default_rng(0)
    planes = (rng.standard_normal((2, 44100)) * 0.1).astype(np.float32)
    spec = packed_spectrum(planes)
    ref = mel_oracle.forward(spec)
    model = Roformer(mel_package, 0, precision)
    got = model.forward(torch.from_numpy(spec.astype(np.float32)).cuda()).cpu().numpy()
    assert got.shape == ref.shape
    snr = snr_db(ref, got)
    print(f"masks {precision}: snr {snr:.1f} dB, max_abs {max_abs(ref, got):.3g}")
    assert snr >= tol_db
    if precision == "f32":
        assert max_abs(ref, got) < 1e-4


def test_config1_waveform_parity(mel_package, mel_oracle):
    """One 8 s chunk (--chunk-samples 352800 --overlap 1): fp32 ≤ 1e-4 / ≥ 80 dB, bf16 ≥ 50 dB."""
    rng = np.random.default_rng(0)
    planes = (rng.standard_normal((2, 352800)) * 0.1).astype(np.float32)
    ref, _ = oracle_runtime.separate(mel_oracle, planes, chunk=352800, overlap=1)
    results = {}
    for precision in ("f32", "bf16"):
        model = Roformer(mel_package, 0, precision)
        got, _ = separate_pcm([model], planes, chunk_samples=352800, overlap=1)
        results[precision] = (snr_db(ref, got), max_abs(ref, got))
        model.close()
    print("config-1 waveform parity:", results)
    assert results["f32"][1] <= 1e-4 and results["f32"][0] >= 80.0
    assert results["bf16"][0] >= 50.0


def test_separate_task_writes_reference_outputs(tmp_path, mel_package):
    """The task API: WAV in, vocals / instrument WAVs + run.json out (runtime_contracts.rs)."""
    import json
    import wave as wavmod
    planes = mono(100000, 0.011)
    inp = str(tmp_path / "in.wav")
    with wavmod.open(inp, "wb") as w:
        w.setnchannels(1)
        w.setsampwidth(2)
        w.setframerate(44100)
        w.writeframes((planes[0] * 32767).astype("<i2").tobytes())
    out = str(tmp_path / "out")
    report = separate(SeparateOptions(inp, mel_package, out, precision="bf16"))
    assert report["backend"] == "cuda" and report["samples_per_channel"] == 100000
    assert report["chunks"] == len(oracle_runtime.chunk_layout(100000, 352800, 4)[3])
    assert report["stems"][1]["origin"] == "residual"
    assert os.path.isfile(os.path.join(out, "vocals.wav"))
    assert os.path.isfile(os.path.join(out, "instrument.wav"))
    assert json.load(open(os.path.join(out, "run.json")))["schema_version"] == 1
    # Cancellation publishes nothing (runtime_contracts.rs:329-343).
    import ctypes
    flag = ctypes.c_int(1)
    with pytest.raises(Exception):
        separate(SeparateOptions(inp, mel_package, str(tmp_path / "cancelled")), cancelled=flag)
    assert not os.path.exists(str(tmp_path / "cancelled"))
