"""Model configuration and manifest schema 1, with the reference's presets.

Mirrors ``crates/ancha-models/src/config.rs`` of the reference: ``ModelConfig`` (13-33) and
its validation (36-121), the presets ``leap_xe`` (123-165), ``mel_karaoke`` (168-171) and
``hyperace_v2`` (173-194), and ``Manifest`` (197-228). Unknown keys are rejected, as
``#[serde(deny_unknown_fields)]`` does.

The Mel karaoke band table is not copied: :func:`mel_band_table` recomputes it from the
Slaney mel filter bank (librosa ``filters.mel`` defaults, ``htk=False``, ``norm='slaney'``),
taking every FFT bin with a positive weight and forcing the first bin of the first band and
the last bin of the last band, as the MelBandRoformer model defines its bands.
"""
from __future__ import annotations

import copy
import json
import re
from dataclasses import dataclass, field, asdict

import numpy as np

FAMILIES = ("bs-roformer", "mel-band-roformer", "hyperace-v2")
STEMS = ("vocals", "instrumental", "lead_vocals")
CONFIG_KEYS = ("family", "dim", "depth", "heads", "head_dim", "ff_mult", "mask_depth",
               "mask_expansion", "sample_rate", "n_fft", "hop", "chunk_samples", "overlap",
               "zero_dc", "stems", "bands")
MANIFEST_KEYS = ("schema_version", "model_id", "weights_sha256", "checkpoint_sha256",
                 "source_url", "forward_revision", "weight_license", "config")


class ConfigError(ValueError):
    """A manifest or configuration that schema 1 rejects."""


def _hz_to_mel(f):
    f = np.asarray(f, dtype=np.float64)
    f_sp = 200.0 / 3.0
    min_log_hz, min_log_mel, logstep = 1000.0, 1000.0 / f_sp, np.log(6.4) / 27.0
    return np.where(f >= min_log_hz,
                    min_log_mel + np.log(np.maximum(f, 1e-10) / min_log_hz) / logstep,
                    f / f_sp)


def _mel_to_hz(m):
    m = np.asarray(m, dtype=np.float64)
    f_sp = 200.0 / 3.0
    min_log_hz, min_log_mel, logstep = 1000.0, 1000.0 / f_sp, np.log(6.4) / 27.0
    return np.where(m >= min_log_mel, min_log_hz * np.exp(logstep * (m - min_log_mel)), f_sp * m)


def mel_band_table(sample_rate: int = 44100, n_fft: int = 2048, bands: int = 60):
    """FFT-bin membership of ``bands`` Slaney mel filters (bins with positive weight)."""
    freqs = np.fft.rfftfreq(n_fft, 1.0 / sample_rate)
    mel_f = _mel_to_hz(np.linspace(_hz_to_mel(0.0), _hz_to_mel(sample_rate / 2.0), bands + 2))
    fdiff = np.diff(mel_f)
    ramps = mel_f[:, None] - freqs[None, :]
    member = np.zeros((bands, freqs.size), dtype=bool)
    for i in range(bands):
        lower = -ramps[i] / fdiff[i]
        upper = ramps[i + 2] / fdiff[i + 1]
        member[i] = np.maximum(0.0, np.minimum(lower, upper)) > 0
    member[0, 0] = True
    member[-1, -1] = True
    return [[int(b) for b in np.nonzero(row)[0]] for row in member]


def _contiguous(counts):
    bands, offset = [], 0
    for n in counts:
        bands.append(list(range(offset, offset + n)))
        offset += n
    return bands


@dataclass
class ModelConfig:
    family: str
    dim: int
    depth: int
    heads: int
    head_dim: int
    ff_mult: int
    mask_depth: int
    mask_expansion: int
    sample_rate: int
    n_fft: int
    hop: int
    chunk_samples: int
    overlap: int
    zero_dc: bool
    stems: list = field(default_factory=list)
    bands: list = field(default_factory=list)

    # -- presets (config.rs:123-194) ------------------------------------------------------
    @classmethod
    def leap_xe(cls, instrumental: bool = False) -> "ModelConfig":
        counts = [2] * 24 + [4] * 36 + [12] * 16 + [24] * 8 + [48] * 4 + [128, 129]
        return cls("bs-roformer", 256, 16, 8, 64, 4, 2, 4, 44100, 2048, 512, 881559, 2, True,
                   ["instrumental" if instrumental else "vocals"], _contiguous(counts))

    @classmethod
    def mel_karaoke(cls) -> "ModelConfig":
        return cls("mel-band-roformer", 384, 6, 8, 64, 4, 2, 4, 44100, 2048, 441, 352800, 4,
                   True, ["lead_vocals"], mel_band_table(44100, 2048, 60))

    @classmethod
    def hyperace_v2(cls, instrumental: bool = False) -> "ModelConfig":
        c = cls.leap_xe(instrumental)
        c.family, c.depth, c.chunk_samples, c.overlap, c.zero_dc = \
            "hyperace-v2", 12, 960000, 4, False
        c.bands = _contiguous([2] * 24 + [4] * 12 + [12] * 8 + [24] * 8 + [48] * 8 + [128, 129])
        return c

    @classmethod
    def bs_roformer_512(cls) -> "ModelConfig":
        """BS-RoFormer dim 512, depth 12, 8×64 heads over the 62-band HyperACE partition."""
        c = cls.hyperace_v2(False)
        c.family, c.dim, c.depth, c.chunk_samples, c.overlap, c.zero_dc = \
            "bs-roformer", 512, 12, 352800, 2, True
        return c

    # -- schema ---------------------------------------------------------------------------
    def validate(self) -> None:
        """Reject what ``ModelConfig::validate`` rejects (config.rs:36-121)."""
        def ensure(ok, msg):
            if not ok:
                raise ConfigError(msg)
        ensure(self.family in FAMILIES, "unknown family")
        ensure(0 < self.dim <= 4096 and 0 < self.depth <= 64, "invalid model dimensions")
        ensure(0 < self.heads <= 64 and 0 < self.head_dim <= 256 and self.head_dim % 2 == 0,
               "invalid attention dimensions")
        ensure(0 < self.ff_mult <= 16 and 0 < self.mask_depth <= 8
               and 0 < self.mask_expansion <= 16, "invalid MLP dimensions")
        ensure(self.sample_rate == 44100 and self.n_fft == 2048 and 1 <= self.hop <= 1024,
               "schema 1 requires 44100 Hz, FFT 2048 and hop <= 1024")
        ensure(self.n_fft // 2 < self.chunk_samples <= 44100 * 60 and 0 < self.overlap <= 16,
               "invalid chunk settings")
        ensure(0 < len(self.stems) <= 2 and all(s in STEMS for s in self.stems),
               "invalid stem labels")
        ensure(len(self.stems) == 1 or self.stems[0] != self.stems[1], "duplicate stems")
        ensure("lead_vocals" not in self.stems
               or (self.family == "mel-band-roformer" and len(self.stems) == 1),
               "lead vocals require a single-head Mel karaoke model")
        ensure(2 <= len(self.bands) <= 256, "invalid band count")
        bins = self.n_fft // 2 + 1
        coverage = [0] * bins
        for band in self.bands:
            ensure(len(band) > 0 and all(a < b for a, b in zip(band, band[1:])),
                   "bands must be nonempty and strictly ordered")
            for f in band:
                ensure(0 <= f < bins, "band index out of range")
                coverage[f] += 1
        ensure(all(n > 0 for n in coverage), "bands leave uncovered FFT bins")
        if self.family != "mel-band-roformer":
            ensure(all(n == 1 for n in coverage), "BS bands must partition the frequency axis")
            ensure([f for b in self.bands for f in b] == list(range(bins)),
                   "BS bands must be contiguous and in frequency order")
        if self.family == "hyperace-v2":
            ensure(self.dim == 256 and len(self.bands) == 62 and len(self.stems) == 1,
                   "HyperACE v2 requires dim=256, 62 bands and one stem")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        unknown = set(d) - set(CONFIG_KEYS)
        missing = set(CONFIG_KEYS) - set(d)
        if unknown or missing:
            raise ConfigError(f"config keys: unknown {sorted(unknown)}, missing {sorted(missing)}")
        return cls(**copy.deepcopy(d))


_HEX64 = re.compile(r"^[0-9a-fA-F]{64}$")


@dataclass
class Manifest:
    schema_version: int
    model_id: str
    weights_sha256: str
    checkpoint_sha256: str
    source_url: str
    forward_revision: str
    weight_license: str
    config: ModelConfig

    def validate(self) -> None:
        """``Manifest::validate`` (config.rs:210-228)."""
        if self.schema_version != 1:
            raise ConfigError("unsupported model package schema")
        if not self.model_id:
            raise ConfigError("model ID is empty")
        for digest in (self.weights_sha256, self.checkpoint_sha256):
            if not _HEX64.match(digest or ""):
                raise ConfigError("invalid SHA256")
        self.config.validate()

    def to_dict(self) -> dict:
        d = asdict(self)
        d["config"] = self.config.to_dict()
        return d

    def dumps(self) -> str:
        return json.dumps(self.to_dict(), indent=2)

    @classmethod
    def from_dict(cls, d: dict) -> "Manifest":
        unknown = set(d) - set(MANIFEST_KEYS)
        missing = set(MANIFEST_KEYS) - set(d)
        if unknown or missing:
            raise ConfigError(f"manifest keys: unknown {sorted(unknown)}, missing {sorted(missing)}")
        d = dict(d)
        d["config"] = ModelConfig.from_dict(d["config"])
        return cls(**d)

    @classmethod
    def load(cls, package: str) -> "Manifest":
        import os
        with open(os.path.join(package, "manifest.json")) as fh:
            m = cls.from_dict(json.load(fh))
        m.validate()
        return m
