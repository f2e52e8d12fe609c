"""Synthetic RoFormer model packages (``manifest.json`` + ``model.safetensors``).

There are no real checkpoints offline, so tests and benchmarks write packages with
synthetic weights under the reference's schema 1 and key names (the PyTorch / MSST names
the reference's strict loader consumes, ``crates/ancha-models/src/network.rs:89-211`` and
``roformer.rs:205-409``).

* :func:`tiny_package` / :func:`kernel_package` reproduce the deterministic fixtures of the
  reference's ``tests/support/mod.rs:12-157`` (gamma ``0.75 + 0.25·(i % 3)``, RoPE freqs
  ``[1, 0.01, …]``, every other value ``((i % 17) − 8)·1e-3``).
* :func:`seeded_package` writes the benchmark model: every Linear weight and bias drawn from
  N(0, std) with numpy's PCG64 generator seeded with ``seed``, tensors filled in sorted key
  order; norm gammas are 1 and RoPE freqs are ``10000^(-2i/head_dim)``.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

from .config import Manifest, ModelConfig


def package_keys(c: ModelConfig):
    """``(key, shape)`` of every tensor a package of config ``c`` holds."""
    dim, inner = c.dim, c.heads * c.head_dim
    hidden, mask = c.dim * c.ff_mult, c.dim * c.mask_expansion
    mel = c.family == "mel-band-roformer"
    keys = []
    for band, bins in enumerate(c.bands):
        width = len(bins) * 4
        p = f"band_split.to_features.{band}"
        keys += [(f"{p}.0.gamma", (width,)), (f"{p}.1.weight", (dim, width)),
                 (f"{p}.1.bias", (dim,))]
    hidden_layers = c.mask_depth if mel else c.mask_depth - 1
    for stem in range(len(c.stems)):
        for band, bins in enumerate(c.bands):
            width = len(bins) * 4
            p = f"mask_estimators.{stem}.to_freqs.{band}.0"
            sizes = [dim] + [mask] * hidden_layers
            for layer in range(hidden_layers):
                keys += [(f"{p}.{layer * 2}.weight", (sizes[layer + 1], sizes[layer])),
                         (f"{p}.{layer * 2}.bias", (sizes[layer + 1],))]
            last = hidden_layers * 2
            keys += [(f"{p}.{last}.weight", (2 * width, sizes[-1])),
                     (f"{p}.{last}.bias", (2 * width,))]
    for i in range(c.depth):
        for axis in range(2):
            p = f"layers.{i}.{axis}"
            a = f"{p}.layers.0.0"
            f = f"{p}.layers.0.1.net"
            keys += [(f"{a}.norm.gamma", (dim,)), (f"{a}.to_qkv.weight", (3 * inner, dim)),
                     (f"{a}.to_gates.weight", (c.heads, dim)), (f"{a}.to_gates.bias", (c.heads,)),
                     (f"{a}.to_out.0.weight", (dim, inner)),
                     (f"{a}.rotary_embed.freqs", (c.head_dim // 2,)),
                     (f"{f}.0.gamma", (dim,)), (f"{f}.1.weight", (hidden, dim)),
                     (f"{f}.1.bias", (hidden,)), (f"{f}.4.weight", (dim, hidden)),
                     (f"{f}.4.bias", (dim,))]
            if mel:
                keys.append((f"{p}.norm.gamma", (dim,)))
    if not mel:
        keys.append(("final_norm.gamma", (dim,)))
    return keys


def write_safetensors(path: str, tensors: dict) -> None:
    """Minimal F32 safetensors writer: 8-byte header length, JSON header, raw data."""
    names = sorted(tensors)
    header, offset = {}, 0
    for name in names:
        a = tensors[name]
        n = a.size * 4
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [offset, offset + n]}
        offset += n
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * ((8 - len(blob) % 8) % 8)
    with open(path, "wb") as fh:
        fh.write(len(blob).to_bytes(8, "little"))
        fh.write(blob)
        for name in names:
            fh.write(np.ascontiguousarray(tensors[name], dtype="<f4").tobytes())


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for block in iter(lambda: fh.read(1 << 22), b""):
            h.update(block)
    return h.hexdigest()


def _finish(directory: str, c: ModelConfig, tensors: dict, model_id: str) -> Manifest:
    os.makedirs(directory, exist_ok=True)
    weights = os.path.join(directory, "model.safetensors")
    write_safetensors(weights, tensors)
    m = Manifest(1, model_id, sha256_file(weights), "0" * 64, "original synthetic tensors",
                 "synthetic schema-1", "MIT", c)
    m.validate()
    with open(os.path.join(directory, "manifest.json"), "w") as fh:
        fh.write(m.dumps())
    return m


def fixture_config(family: str, kernel: bool = False) -> ModelConfig:
    """The reference's test fixture config (``tests/support/mod.rs:27-58``)."""
    c = ModelConfig.leap_xe(False)
    c.family = family
    c.dim, c.depth, c.heads, c.head_dim, c.ff_mult = 4, 1, 1, 4, 1
    c.mask_depth, c.mask_expansion, c.chunk_samples, c.overlap = 2, 1, 4096, 2
    if family == "bs-roformer":
        c.bands = [list(range(0, 300)), list(range(300, 700)), list(range(700, 1000)),
                   list(range(1000, 1025))]
    else:
        c.bands = [list(range(0, 400)), list(range(300, 900)), list(range(625, 1025))]
        c.stems = ["vocals", "instrumental"]
    if kernel:
        c.dim, c.heads, c.head_dim, c.ff_mult = 128, 2, 64, 4
    return c


def deterministic_package(directory: str, c: ModelConfig, model_id="synthetic-ci-fixture"):
    tensors = {}
    for key, shape in package_keys(c):
        i = np.arange(int(np.prod(shape)))
        if key.endswith("gamma"):
            v = 0.75 + (i % 3).astype(np.float32) * 0.25
        elif key.endswith("freqs"):
            v = np.where(i == 0, 1.0, 0.01)
        else:
            v = ((i % 17).astype(np.float32) - 8.0) * 0.001
        tensors[key] = np.asarray(v, dtype=np.float32).reshape(shape)
    return _finish(directory, c, tensors, model_id)


def tiny_package(directory: str, family: str) -> Manifest:
    return deterministic_package(directory, fixture_config(family))


def kernel_package(directory: str, family: str) -> Manifest:
    return deterministic_package(directory, fixture_config(family, kernel=True))


def seeded_package(directory: str, c: ModelConfig, seed: int = 0, std: float = 0.02,
                   model_id: str | None = None) -> Manifest:
    rng = np.random.default_rng(seed)
    tensors = {}
    for key, shape in sorted(package_keys(c)):
        if key.endswith("gamma"):
            v = np.ones(shape, dtype=np.float32)
        elif key.endswith("freqs"):
            i = np.arange(shape[0], dtype=np.float64)
            v = (10000.0 ** (-2.0 * i / c.head_dim)).astype(np.float32)
        else:
            v = (rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(std))
            v = v.reshape(shape)
        tensors[key] = v
    fam = {"mel-band-roformer": "mel", "bs-roformer": "bs", "hyperace-v2": "hyperace"}[c.family]
    return _finish(directory, c, tensors, model_id or f"synthetic-{fam}-seed{seed}")
