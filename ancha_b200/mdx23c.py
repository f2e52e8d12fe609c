"""MDX23C (TFC-TDF v3) over the C ABI, mirroring ``Mdx23c::load`` / ``forward``
(``crates/ancha-models/src/mdx23c.rs:372-481``).

:class:`Mdx23c` is a package resident on one GPU; ``forward`` maps a CUDA f32 spectrum
``[batch, 4, bins, frames]`` (L.re, L.im, R.re, R.im) to the predicted stem spectra
``[batch, stems·4, bins, frames]``. :func:`write_package` writes a schema-1 package
(``manifest.json`` + ``model.safetensors``) from host tensors, the layout the reference's
tests build (``crates/ancha-models/tests/support/mdx23c.rs:51-100``).
"""
from __future__ import annotations

import ctypes as C
import json
import os
from typing import Optional

from . import _native as N
from .synthetic import sha256_file, write_safetensors

FORWARD_REVISION = "UVR/5517e0cf0d1acd16a1618eeedec596957523f9e1;lib_v5/tfc_tdf_v3.py"


class Mdx23c:
    """An MDX23C package on one GPU (not re-entrant; one per device and thread)."""

    def __init__(self, package: str, device: int = 0, precision: str = "f16"):
        self.precision = N.PRECISIONS[precision]
        handle = C.c_void_p()
        N.check(N.lib().ancha_mdx23c_load(package.encode(), device, self.precision, C.byref(handle)))
        self._h = handle
        self.device = device
        vals = [C.c_int() for _ in range(7)]
        N.check(N.lib().ancha_mdx23c_info(self._h, *[C.byref(v) for v in vals]))
        (self.bins, self.frames, self.n_fft, self.hop, self.overlap, self.stems,
         self.tensor_count) = (v.value for v in vals)

    def forward(self, spectrum, cancel: Optional[C.c_int] = None):
        """Stem spectra for a CUDA f32 tensor ``[batch, 4, bins, frames]``."""
        import torch
        s = spectrum.contiguous().float()
        if s.dim() != 4 or s.shape[1] != 4 or s.shape[2] != self.bins:
            raise N.AnchaError(N.E_INVALID, "invalid MDX23C spectrum shape")
        b, _, _, frames = s.shape
        out = torch.empty((b, self.stems * 4, self.bins, frames), dtype=torch.float32, device=s.device)
        stream = C.c_void_p(torch.cuda.current_stream(s.device).cuda_stream)
        N.check(N.lib().ancha_mdx23c_forward(self._h, s.data_ptr(), b, frames, out.data_ptr(),
                                             None if cancel is None else C.byref(cancel), stream))
        return out

    def separate_pcm(self, planes, overlap: int = 0, batch: int = 0, cancel: Optional[C.c_int] = None):
        """``mdx23c_runtime::separate`` on host PCM: ``[2, samples]`` f32 → ``([stems, 2, samples],
        seconds)``; chunking, STFT, network, iSTFT and overlap-add all run on this model's GPU."""
        import numpy as np
        x = np.ascontiguousarray(planes, dtype=np.float32)
        if x.ndim != 2 or x.shape[0] != 2:
            raise N.AnchaError(N.E_INVALID, "planes must be [2, samples]")
        out = np.empty((self.stems, 2, x.shape[1]), dtype=np.float32)
        secs = C.c_double()
        fp = C.POINTER(C.c_float)
        N.check(N.lib().ancha_mdx23c_separate_pcm(self._h, x.ctypes.data_as(fp), x.shape[1], overlap, batch,
                                                  None if cancel is None else C.byref(cancel),
                                                  out.ctypes.data_as(fp), C.byref(secs)))
        return out, secs.value

    def close(self) -> None:
        if self._h:
            N.lib().ancha_mdx23c_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OverlapPlan:
    """``OverlapPlan::new`` (src/mdx23c_runtime.rs:84-115) through ``ancha_mdx23c_plan``:
    ``step``, ``border``, ``pad``, ``padded`` and ``chunks`` of a ``samples``-long track."""

    def __init__(self, samples: int, chunk_samples: int, overlap: int):
        vals = [C.c_int64() for _ in range(5)]
        N.check(N.lib().ancha_mdx23c_plan(samples, chunk_samples, overlap, *[C.byref(v) for v in vals]))
        self.samples, self.chunk = samples, chunk_samples
        self.step, self.border, self.pad, self.padded, self.chunks = (v.value for v in vals)

    def intersects(self, start: int) -> bool:
        return start < self.border + self.samples and start + self.chunk > self.border


def write_package(directory: str, config: dict, tensors: dict, model_id: str = "synthetic-mdx23c") -> dict:
    """Write ``model.safetensors`` (F32) and a schema-1 ``manifest.json``; returns the manifest."""
    os.makedirs(directory, exist_ok=True)
    weights = os.path.join(directory, "model.safetensors")
    write_safetensors(weights, tensors)
    manifest = {
        "schema_version": 1,
        "model_id": model_id,
        "weights_sha256": sha256_file(weights),
        "checkpoint_sha256": "0" * 64,
        "source_url": "original synthetic contract",
        "forward_revision": FORWARD_REVISION,
        "weight_license": "MIT synthetic data",
        "config": config,
    }
    with open(os.path.join(directory, "manifest.json"), "w") as fh:
        json.dump(manifest, fh, indent=2)
    return manifest


def inst_voc_hq2() -> dict:
    """The ``Config::inst_voc_hq2`` preset (mdx23c.rs:56-74), the benchmarked MDX23C network."""
    return dict(family="mdx23c", sample_rate=44100, n_fft=8192, hop=1024, bins=4096, frames=256, overlap=8,
                subbands=4, channels=128, growth=128, scales=5, blocks_per_scale=2, bottleneck_factor=4,
                scale=[2, 2], stems=["vocals", "instrumental"])


def tensor_shapes(c: dict) -> dict:
    """Name → shape of every tensor of a package (the key layout of Mdx23c::build,
    mdx23c.rs:379-418)."""
    shapes = {}
    inp = 4 * c["subbands"]

    def norm(p, ch):
        shapes[p + ".weight"] = (ch,)
        shapes[p + ".bias"] = (ch,)

    def blocks(p, ci, co, f):
        fb = f // c["bottleneck_factor"]
        for i in range(c["blocks_per_scale"]):
            q, cin = f"{p}.blocks.{i}", ci if i == 0 else co
            norm(q + ".tfc1.0", cin)
            shapes[q + ".tfc1.2.weight"] = (co, cin, 3, 3)
            norm(q + ".tdf.0", co)
            shapes[q + ".tdf.2.weight"] = (fb, f)
            norm(q + ".tdf.3", co)
            shapes[q + ".tdf.5.weight"] = (f, fb)
            norm(q + ".tfc2.0", co)
            shapes[q + ".tfc2.2.weight"] = (co, co, 3, 3)
            shapes[q + ".shortcut.weight"] = (co, cin, 1, 1)

    shapes["first_conv.weight"] = (c["channels"], inp, 1, 1)
    ch, f = c["channels"], c["bins"] // c["subbands"]
    for i in range(c["scales"]):
        p = f"encoder_blocks.{i}"
        blocks(p + ".tfc_tdf", ch, ch, f)
        norm(p + ".downscale.conv.0", ch)
        shapes[p + ".downscale.conv.2.weight"] = (ch + c["growth"], ch, 2, 2)
        f, ch = f // 2, ch + c["growth"]
    blocks("bottleneck_block", ch, ch, f)
    for i in range(c["scales"]):
        p, co = f"decoder_blocks.{i}", ch - c["growth"]
        f *= 2
        norm(p + ".upscale.conv.0", ch)
        shapes[p + ".upscale.conv.2.weight"] = (ch, co, 2, 2)
        blocks(p + ".tfc_tdf", 2 * co, co, f)
        ch = co
    shapes["final_conv.0.weight"] = (ch, ch + inp, 1, 1)
    shapes["final_conv.2.weight"] = (len(c["stems"]) * inp, ch, 1, 1)
    return shapes


def random_tensors(c: dict, seed: int = 0) -> dict:
    """Seeded synthetic weights: norm gammas 1 + 0.1·N(0, 1), betas 0.1·N(0, 1), matrices
    N(0, 1 / fan_in) (variance-preserving, so activations stay O(1) through the network)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in sorted(tensor_shapes(c).items()):
        if len(shape) == 1:
            base = 1.0 if name.endswith("weight") else 0.0
            out[name] = (base + 0.1 * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        else:
            fan_in = int(np.prod(shape[1:]))
            out[name] = (rng.standard_normal(shape, dtype=np.float32) / np.float32(np.sqrt(fan_in)))
    return out


def forward_flops(c: dict, batch: int, frames: int) -> int:
    """Algorithmic FLOPs of one forward: 2·M·N·K over every convolution (as patch GEMMs),
    TDF Linear and transpose convolution; elementwise work is not counted."""
    inp, g, bn = 4 * c["subbands"], c["growth"], c["bottleneck_factor"]
    f0 = c["bins"] // c["subbands"]
    total = 0

    def blocks(ci, co, t, f):
        nonlocal total
        pos = t * f
        for i in range(c["blocks_per_scale"]):
            cin = ci if i == 0 else co
            total += 2 * pos * co * (cin + 9 * cin + 9 * co)      # shortcut, tfc1, tfc2
            total += 2 * 2 * (co * t) * f * (f // bn)              # the two TDF Linears

    ch, t, f = c["channels"], frames, f0
    total += 2 * (t * f) * ch * inp
    for _ in range(c["scales"]):
        blocks(ch, ch, t, f)
        t, f = t // 2, f // 2
        total += 2 * (t * f) * (ch + g) * 4 * ch
        ch += g
    blocks(ch, ch, t, f)
    for _ in range(c["scales"]):
        co = ch - g
        total += 2 * (t * f) * 4 * co * ch
        t, f = 2 * t, 2 * f
        blocks(2 * co, co, t, f)
        ch = co
    total += 2 * (t * f) * (ch * (ch + inp) + len(c["stems"]) * inp * ch)
    return batch * total
