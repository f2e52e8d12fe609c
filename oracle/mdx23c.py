"""MDX23C (TFC-TDF v3) spectral network in numpy (test oracle only).

Restates the reference's generic CPU path of ``crates/ancha-models/src/mdx23c.rs``:

* configuration checks: ``Config::validate`` (mdx23c.rs:76-122), the ``inst_voc_hq2``
  preset (mdx23c.rs:56-74);
* weight names, shapes and construction order: ``Mdx23c::build`` (mdx23c.rs:379-418),
  ``Block::load`` (mdx23c.rs:243-263), ``Blocks::load`` (mdx23c.rs:277-302);
* forward: ``Mdx23c::forward`` (mdx23c.rs:420-481), ``Block::forward`` (mdx23c.rs:264-274),
  ``Up::forward`` (mdx23c.rs:330-355), ``Preact`` = GELU(InstanceNorm(x)) with epsilon 1e-5
  and the biased spatial variance (mdx23c.rs:200-213, spatial.rs:104-126), ``tdf`` = a
  bias-free Linear over the last (frequency) axis (mdx23c.rs:225-241, weights.rs:104-128:
  stored ``[out, in]``), ``conv2d`` with PyTorch's ``[out, in, kh, kw]`` weights and no bias
  (mdx23c.rs:152-190), the non-overlapping ``ConvTranspose2d`` with kernel = stride = 2
  (spatial.rs:128-150, weights ``[in, out, 2, 2]``).

Activations are NCHW ``[batch, channels, time, frequency]`` inside the network, as in the
reference after its ``swap_dims(2, 3)``. Arithmetic is float64. GELU is the exact erf form.

``fixture_weights`` / ``fixture_input`` restate the closed-form synthetic weights and input
of the reference's golden test (``crates/ancha-models/tests/support/mdx23c.rs:27-78``), whose
PyTorch output is kept in ``tests/golden/mdx23c_tiny.json``.
"""
from __future__ import annotations

import math

import numpy as np

try:
    from scipy.special import erf as _erf
except ImportError:  # pragma: no cover
    _erf = np.vectorize(math.erf)

CONFIG_KEYS = ("family", "sample_rate", "n_fft", "hop", "bins", "frames", "overlap", "subbands",
               "channels", "growth", "scales", "blocks_per_scale", "bottleneck_factor", "scale",
               "stems")


def inst_voc_hq2() -> dict:
    """The ``Config::inst_voc_hq2`` preset (mdx23c.rs:56-74)."""
    return dict(family="mdx23c", sample_rate=44100, n_fft=8192, hop=1024, bins=4096, frames=256,
                overlap=8, subbands=4, channels=128, growth=128, scales=5, blocks_per_scale=2,
                bottleneck_factor=4, scale=[2, 2], stems=["vocals", "instrumental"])


def chunk_samples(c: dict) -> int:
    return c["hop"] * (c["frames"] - 1)


def validate(c: dict) -> None:
    """``Config::validate`` (mdx23c.rs:76-122); raises ValueError."""
    if set(c) != set(CONFIG_KEYS) or c["family"] != "mdx23c":
        raise ValueError("not an MDX23C config")
    n_fft, hop = c["n_fft"], c["hop"]
    if not (c["sample_rate"] == 44100 and 32 <= n_fft <= 8192 and n_fft % 2 == 0 and 0 < hop <= n_fft // 2):
        raise ValueError("MDX23C requires stereo 44100 Hz and a valid centered STFT")
    if not (1 <= c["scales"] <= 6 and list(c["scale"]) == [2, 2]):
        raise ValueError("MDX23C supports 1..=6 scales with 2x2 down/up sampling")
    factor = 1 << c["scales"]
    sub, bins, frames = c["subbands"], c["bins"], c["frames"]
    if not (1 <= sub <= 16 and 0 < bins <= n_fft // 2 + 1 and bins % (sub * factor) == 0
            and factor <= frames <= 2048 and frames % factor == 0):
        raise ValueError("MDX23C frequency/time dimensions must survive all encoder scales")
    ch, g = c["channels"], c["growth"]
    if not (1 <= ch <= 1024 and 1 <= g <= 1024 and ch + c["scales"] * g <= 2048
            and 1 <= c["blocks_per_scale"] <= 4 and 1 <= c["bottleneck_factor"] <= 16):
        raise ValueError("invalid MDX23C network size")
    bottom = bins // sub // factor
    if not (bottom >= c["bottleneck_factor"] and (frames // factor) * bottom > 1):
        raise ValueError("MDX23C bottleneck is too small for Linear or InstanceNorm")
    if not (n_fft // 2 < chunk_samples(c) <= 44100 * 60 and 1 <= c["overlap"] <= 16):
        raise ValueError("invalid MDX23C context")
    if list(c["stems"]) != ["vocals", "instrumental"]:
        raise ValueError("MDX23C schema 1 requires two native heads in vocals/instrumental order")


def weight_shapes(c: dict) -> dict:
    """Every tensor the network reads, name → shape, in ``Mdx23c::build`` terms
    (mdx23c.rs:379-418; block keys mdx23c.rs:243-263)."""
    shapes = {}
    inp = 4 * c["subbands"]

    def norm(p, ch):
        shapes[p + ".weight"] = (ch,)
        shapes[p + ".bias"] = (ch,)

    def blocks(p, ci, co, f):
        bn = c["bottleneck_factor"]
        for i in range(c["blocks_per_scale"]):
            q = f"{p}.blocks.{i}"
            cin = ci if i == 0 else co
            norm(q + ".tfc1.0", cin)
            shapes[q + ".tfc1.2.weight"] = (co, cin, 3, 3)
            norm(q + ".tdf.0", co)
            shapes[q + ".tdf.2.weight"] = (f // bn, f)
            norm(q + ".tdf.3", co)
            shapes[q + ".tdf.5.weight"] = (f, f // bn)
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
        f //= 2
        ch += c["growth"]
    blocks("bottleneck_block", ch, ch, f)
    for i in range(c["scales"]):
        p = f"decoder_blocks.{i}"
        co = ch - c["growth"]
        f *= 2
        norm(p + ".upscale.conv.0", ch)
        shapes[p + ".upscale.conv.2.weight"] = (ch, co, 2, 2)
        blocks(p + ".tfc_tdf", co * 2, co, f)
        ch = co
    shapes["final_conv.0.weight"] = (ch, ch + inp, 1, 1)
    shapes["final_conv.2.weight"] = (len(c["stems"]) * inp, ch, 1, 1)
    return shapes


def fixture_weights(names_shapes) -> dict:
    """Synthetic weights of the golden test (tests/support/mdx23c.rs:51-66): with
    seed = Σ bytes(name) mod 97 and phase = (i + 1)·0.17 + seed·0.11, a 1-D ``…weight``
    (norm gamma) is 1 + 0.03·sin(phase), everything else 0.02·sin(phase); f64 → f32."""
    out = {}
    for name, shape in names_shapes:
        seed = sum(name.encode()) % 97
        i = np.arange(int(np.prod(shape)), dtype=np.float64)
        phase = (i + 1) * 0.17 + seed * 0.11
        if len(shape) == 1 and name.endswith("weight"):
            v = 1.0 + 0.03 * np.sin(phase)
        else:
            v = 0.02 * np.sin(phase)
        out[name] = v.astype(np.float32).reshape(shape)
    return out


def fixture_input(shape) -> np.ndarray:
    """Input of the golden test (tests/support/mdx23c.rs:27-31): 0.3·sin((i + 1)·0.071)."""
    i = np.arange(int(np.prod(shape)), dtype=np.float64)
    return (0.3 * np.sin((i + 1) * 0.071)).astype(np.float32).reshape(shape)


def gelu(x):
    return 0.5 * x * (1.0 + _erf(x / math.sqrt(2.0)))


def instance_norm(x, gamma, beta, eps=1e-5):
    """Per (batch, channel) over the spatial axes, biased variance (spatial.rs:104-126)."""
    mean = x.mean(axis=(2, 3), keepdims=True)
    c = x - mean
    var = (c * c).mean(axis=(2, 3), keepdims=True)
    return c / np.sqrt(var + eps) * gamma.reshape(1, -1, 1, 1) + beta.reshape(1, -1, 1, 1)


def preact(w, p, x):
    return gelu(instance_norm(x, w[p + ".weight"].astype(np.float64), w[p + ".bias"].astype(np.float64)))


def conv2d(x, weight, stride=(1, 1), padding=(0, 0)):
    """Bias-free 2-D convolution, PyTorch ``[out, in, kh, kw]`` weights."""
    b, ci, h, wd = x.shape
    co, wi, kh, kw = weight.shape
    if wi != ci:
        raise ValueError("conv2d channel mismatch")
    ph, pw = padding
    sh, sw = stride
    xp = np.pad(x, ((0, 0), (0, 0), (ph, ph), (pw, pw)))
    oh = (h + 2 * ph - kh) // sh + 1
    ow = (wd + 2 * pw - kw) // sw + 1
    out = np.zeros((b, co, oh, ow))
    wt = weight.astype(np.float64)
    for ky in range(kh):
        for kx in range(kw):
            patch = xp[:, :, ky:ky + sh * (oh - 1) + 1:sh, kx:kx + sw * (ow - 1) + 1:sw]
            out += np.einsum("bchw,oc->bohw", patch, wt[:, :, ky, kx])
    return out


def conv_transpose2x2(x, weight):
    """ConvTranspose2d with kernel = stride = 2, no padding: every input position writes its
    own 2×2 output block (spatial.rs:128-150); weights ``[in, out, 2, 2]``."""
    b, ci, h, wd = x.shape
    wi, co, kh, kw = weight.shape
    if wi != ci:
        raise ValueError("conv_transpose channel mismatch")
    y = np.einsum("bihw,ioyx->bohywx", x, weight.astype(np.float64))
    return y.reshape(b, co, h * kh, wd * kw)


def tdf(w, name, x):
    """Bias-free Linear over the last axis; weight stored ``[out, in]``."""
    return x @ w[name].astype(np.float64).T


def block(w, p, x):
    """``Block::forward`` (mdx23c.rs:264-274)."""
    skip = conv2d(x, w[p + ".shortcut.weight"])
    x = conv2d(preact(w, p + ".tfc1.0", x), w[p + ".tfc1.2.weight"], padding=(1, 1))
    y = tdf(w, p + ".tdf.2.weight", preact(w, p + ".tdf.0", x))
    y = tdf(w, p + ".tdf.5.weight", preact(w, p + ".tdf.3", y))
    return conv2d(preact(w, p + ".tfc2.0", x + y), w[p + ".tfc2.2.weight"], padding=(1, 1)) + skip


def blocks(w, c, p, x):
    for i in range(c["blocks_per_scale"]):
        x = block(w, f"{p}.blocks.{i}", x)
    return x


def forward(c: dict, w: dict, spectrum: np.ndarray) -> np.ndarray:
    """``Mdx23c::forward`` (mdx23c.rs:420-481): ``[b, 4, bins, frames]`` (L.re, L.im, R.re,
    R.im) → ``[b, stems·4, bins, frames]`` (spectra, not masks)."""
    b, ch4, f, t = spectrum.shape
    factor = 1 << c["scales"]
    if not (0 < b <= 4 and ch4 == 4 and f == c["bins"] and t >= factor and t % factor == 0):
        raise ValueError("invalid MDX23C spectrum shape")
    sub = c["subbands"]
    mix = spectrum.astype(np.float64).reshape(b, 4 * sub, f // sub, t)
    first = conv2d(mix, w["first_conv.weight"])
    x = first.transpose(0, 1, 3, 2)
    skips = []
    for i in range(c["scales"]):
        p = f"encoder_blocks.{i}"
        x = blocks(w, c, p + ".tfc_tdf", x)
        skips.append(x)
        x = conv2d(preact(w, p + ".downscale.conv.0", x), w[p + ".downscale.conv.2.weight"], stride=(2, 2))
    x = blocks(w, c, "bottleneck_block", x)
    for i in range(c["scales"]):
        p = f"decoder_blocks.{i}"
        x = conv_transpose2x2(preact(w, p + ".upscale.conv.0", x), w[p + ".upscale.conv.2.weight"])
        skip = skips.pop()
        if x.shape[2:] != skip.shape[2:]:
            raise ValueError("MDX23C decoder skip shape mismatch")
        x = blocks(w, c, p + ".tfc_tdf", np.concatenate([x, skip], axis=1))
    x = x.transpose(0, 1, 3, 2) * first
    x = conv2d(np.concatenate([mix, x], axis=1), w["final_conv.0.weight"])
    x = conv2d(gelu(x), w["final_conv.2.weight"])
    return x.reshape(b, len(c["stems"]) * 4, f, t)


class OverlapPlan:
    """UVR chunking of ``mdx23c_runtime.rs:73-132``: step = chunk / overlap, a left border of
    chunk − step zeros and a right pad that makes the padded length a whole number of steps
    (Python modulo semantics), chunks starting every step; the overlap-add divides by the
    constant ``overlap``."""

    def __init__(self, length: int, chunk: int, overlap: int):
        if not (length > 0 and chunk > 0 and 1 <= overlap <= 16 and overlap <= chunk):
            raise ValueError("invalid MDX23C overlap plan")
        step = chunk // overlap
        left, right = length % step, chunk % step
        remainder = left - right if left >= right else step - (right - left)
        self.chunk, self.step, self.length = chunk, step, length
        self.pad = step - remainder
        self.border = chunk - step
        self.padded = length + self.pad + 2 * self.border
        if self.padded > 2 ** 63 - 1:
            raise ValueError("MDX23C padded length overflow")
        if self.padded < chunk:
            raise ValueError("insufficient MDX23C padding")
        self.chunks = (self.padded - chunk) // step + 1

    def intersects(self, start: int) -> bool:
        return start < self.border + self.length and start + self.chunk > self.border

    def window(self, planes: np.ndarray, start: int) -> np.ndarray:
        """Samples [start, start + chunk) of the zero-bordered signal (mdx23c_runtime.rs:116-132)."""
        out = np.zeros(planes.shape[:-1] + (self.chunk,), dtype=planes.dtype)
        lo, hi = max(start, self.border), min(start + self.chunk, self.border + self.length)
        if hi > lo:
            out[..., lo - start:hi - start] = planes[..., lo - self.border:hi - self.border]
        return out


def pack(stft, planes: np.ndarray, bins: int) -> np.ndarray:
    """``spectral::pack`` with no low-bin suppression (src/spectral.rs:5-36): stereo planes
    ``[2, samples]`` → ``[4, bins, frames]`` = (L.re, L.im, R.re, R.im)."""
    frames = planes.shape[1] // stft.hop + 1
    out = np.empty((4, bins, frames))
    for ch in range(2):
        spec = stft.forward(planes[ch])  # [frames, n_fft / 2 + 1]
        out[2 * ch] = spec[:, :bins].real.T
        out[2 * ch + 1] = spec[:, :bins].imag.T
    return out


def unpack(stft, packed: np.ndarray, length: int) -> np.ndarray:
    """``spectral::unpack`` (src/spectral.rs:38-76): ``[4, bins, frames]`` → ``[2, length]``;
    bins past ``bins`` are zero, Im of DC and Nyquist dropped, no DC zeroing."""
    _, bins, frames = packed.shape
    full = stft.n_fft // 2 + 1
    out = []
    for ch in range(2):
        spec = np.zeros((frames, full), dtype=np.complex128)
        spec[:, :bins] = packed[2 * ch].T + 1j * packed[2 * ch + 1].T
        out.append(stft.inverse(spec, length, False))
    return np.stack(out)


def separate(c: dict, w: dict, planes: np.ndarray, overlap: int | None = None, optimized: bool = True) -> np.ndarray:
    """``mdx23c_runtime::separate`` without file I/O (src/mdx23c_runtime.rs:135-248): UVR
    chunks (zero borders) → centred STFT → forward → iSTFT per stem → rectangular overlap-add
    / overlap. ``optimized`` skips chunks that lie entirely in the zero borders, as the
    reference does with its default options. Returns ``[stems, 2, samples]``."""
    from .dsp import Stft
    n = planes.shape[1]
    ov = overlap or c["overlap"]
    plan = OverlapPlan(n, chunk_samples(c), ov)
    stft = Stft(c["n_fft"], c["hop"])
    stems = len(c["stems"])
    out = np.zeros((stems, 2, n))
    for i in range(plan.chunks):
        start = i * plan.step
        if optimized and not plan.intersects(start):
            continue
        spec = pack(stft, plan.window(planes, start), c["bins"])
        if spec.shape[2] != c["frames"]:
            raise ValueError("MDX23C STFT frame count mismatch")
        y = forward(c, w, spec[None])[0]
        lo, hi = max(start, plan.border), min(start + plan.chunk, plan.border + n)
        for s in range(stems):
            wave = unpack(stft, y[4 * s:4 * s + 4], plan.chunk)
            out[s, :, lo - plan.border:hi - plan.border] += wave[:, lo - start:hi - start]
    return out / ov
