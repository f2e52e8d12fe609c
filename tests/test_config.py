"""Manifest / config schema 1 (config.rs:36-228) and the regenerated Mel band table."""
import hashlib
import json
import os

import pytest

from ancha_b200.config import ConfigError, Manifest, ModelConfig, mel_band_table
from ancha_b200 import synthetic

# The reference project's checkout, when the environment names one (ANCHA_REFERENCE_ROOT).
REFERENCE_MEL = os.path.join(os.environ.get("ANCHA_REFERENCE_ROOT", "/nonexistent"), "configs", "mel-karaoke.json")
# SHA-256 of json.dumps(bands) for the 60-band Slaney table (equal to the bands of the
# reference's configs/mel-karaoke.json; compared with the file itself where it is available).
MEL_SHA = "9a633e38e5ac65de299c8e854842a837f9778a5053e4797fc6e14be0bec02f86"


def test_mel_band_table_matches_reference():
    bands = mel_band_table(44100, 2048, 60)
    assert len(bands) == 60 and sum(map(len, bands)) == 1979
    assert hashlib.sha256(json.dumps(bands).encode()).hexdigest() == MEL_SHA
    if os.path.exists(REFERENCE_MEL):
        assert bands == json.load(open(REFERENCE_MEL))["bands"]


def test_presets_validate_and_match_reference_shapes():
    # model_contracts.rs:90-138
    leap = ModelConfig.leap_xe(False)
    leap.validate()
    assert len(leap.bands) == 90
    k = ModelConfig.mel_karaoke()
    k.validate()
    assert (k.dim, k.depth, len(k.bands), k.chunk_samples, k.overlap) == (384, 6, 60, 352800, 4)
    assert k.stems == ["lead_vocals"]
    bs = ModelConfig.bs_roformer_512()
    bs.validate()
    assert len(bs.bands) == 62 and bs.dim == 512 and bs.depth == 12


@pytest.mark.parametrize("mutate", [
    lambda c: c.bands[0].clear(),
    lambda c: c.bands[0].append(1),
    lambda c: setattr(c, "stems", ["vocals", "vocals"]),
    lambda c: setattr(c, "stems", ["lead_vocals"]),
    lambda c: setattr(c, "n_fft", 4096),
])
def test_config_rejections(mutate):
    c = ModelConfig.leap_xe(False)
    mutate(c)
    with pytest.raises(ConfigError):
        c.validate()


def test_manifest_rejections():
    m = Manifest(1, "leap-xe-voc", "0" * 64, "0" * 64, "fixture", "fixture", "fixture",
                 ModelConfig.leap_xe(False))
    m.validate()
    m.schema_version = 2
    with pytest.raises(ConfigError):
        m.validate()
    m.schema_version = 1
    m.weights_sha256 = "bad"
    with pytest.raises(ConfigError):
        m.validate()
    d = m.to_dict()
    d["unknown"] = True
    with pytest.raises(ConfigError):
        Manifest.from_dict(d)


def test_synthetic_packages_round_trip(tmp_path):
    m = synthetic.tiny_package(str(tmp_path / "bs"), "bs-roformer")
    assert Manifest.load(str(tmp_path / "bs")).weights_sha256 == m.weights_sha256
    from safetensors.numpy import load_file
    w = load_file(str(tmp_path / "bs" / "model.safetensors"))
    assert set(w) == {k for k, _ in synthetic.package_keys(m.config)}
    assert w["band_split.to_features.0.0.gamma"][:3].tolist() == [0.75, 1.0, 1.25]
