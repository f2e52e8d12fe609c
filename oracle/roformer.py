"""Mel-Band / BS-RoFormer forward in numpy (test oracle only).

Restates the reference's generic (non-kernel) CPU path:

* load-time folding: ``crates/ancha-models/src/network.rs:89-278`` (band split with
  ``sqrt(width)·gamma`` folded, mask heads split into GLU value / gate halves),
  ``roformer.rs:205-256`` (q / k / v / gate projections with ``sqrt(dim)·gamma`` folded),
  ``roformer.rs:381-409`` (feed-forward with the norm folded), ``weights.rs:149-176``
  (``folded_linear``: ``W'[i][o] = W[o][i]·input_scale[i]``);
* forward: ``network.rs:301-400`` (band split, axial loop, final norm, mask heads and the
  overlapping-band scatter-add divided by coverage), ``roformer.rs:258-270`` (attention
  block), ``roformer.rs:439-459`` (transformer), ``roformer.rs:16-55`` (``unit_norm``,
  ``SourceNorm``), ``roformer.rs:150-187`` and ``274-309`` (interleaved RoPE tables, the
  query table carrying ``1/sqrt(head_dim)``).

Layouts follow the reference: the spectrum is ``[frames, rows·2]`` packed as
``(frame, bin·2 + channel, re/im)``; masks are ``[stems, rows, re/im, frames]`` with
``rows = bins·2``. GELU is the exact erf form (Burn ``gelu``).
"""
from __future__ import annotations

import json
import math
import os

import numpy as np
from safetensors.numpy import load_file

try:  # scipy's erf is vectorised; math.erf is the fallback.
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)


def unit_norm(x: np.ndarray) -> np.ndarray:
    """``x / max(||x||_2, 1e-12)`` over the last axis (roformer.rs:16-24)."""
    n = np.sqrt((x * x).sum(axis=-1, keepdims=True))
    return x / np.maximum(n, 1e-12)


def gelu(x: np.ndarray) -> np.ndarray:
    return 0.5 * x * (1.0 + _erf(x / math.sqrt(2.0)))


def sigmoid(x: np.ndarray) -> np.ndarray:
    return 1.0 / (1.0 + np.exp(-x))


def rope_tables(freqs: np.ndarray, tokens: int, scale: float):
    """Per-token ``cos`` / signed ``sin`` of one head, ``[tokens, head_dim]`` (roformer.rs:155-175).

    The angle is ``t·f`` rounded to f32 as the reference computes it; sine and cosine are
    then taken in float64.
    """
    f = np.asarray(freqs, dtype=np.float32)
    t = np.arange(tokens, dtype=np.float32)[:, None]
    ang = (t * f[None, :]).astype(np.float64)
    c, s = np.cos(ang) * scale, np.sin(ang) * scale
    cos = np.repeat(c, 2, axis=1)
    sin = np.stack([-s, s], axis=2).reshape(tokens, -1)
    return cos, sin


def rope_apply(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, heads: int) -> np.ndarray:
    """``x·cos + swap_pairs(x)·sin`` on ``[groups, tokens, heads·d]`` (roformer.rs:177-186)."""
    g, n, w = x.shape
    d = w // heads
    xh = x.reshape(g, n, heads, d)
    sw = xh.reshape(g, n, heads, d // 2, 2)[..., ::-1].reshape(g, n, heads, d)
    return (xh * cos[None, :, None, :] + sw * sin[None, :, None, :]).reshape(g, n, w)


class Transformer:
    """One axial transformer (``roformer.rs:374-459``) with its folded weights."""

    def __init__(self, w: dict, p: str, c: dict, normalized: bool, dtype, wround=None):
        dim, heads, hd = c["dim"], c["heads"], c["head_dim"]
        inner = heads * hd
        root = math.sqrt(dim)
        a = f"{p}.layers.0.0"
        norm = w[f"{a}.norm.gamma"].astype(np.float64) * root
        qkv = w[f"{a}.to_qkv.weight"].astype(np.float64)          # [3·inner, dim]
        self.wq = (qkv[:inner] * norm[None, :]).T.astype(dtype)      # [dim, inner]
        self.wk = (qkv[inner:2 * inner] * norm[None, :]).T.astype(dtype)
        self.wv = (qkv[2 * inner:] * norm[None, :]).T.astype(dtype)
        self.wg = (w[f"{a}.to_gates.weight"].astype(np.float64) * norm[None, :]).T.astype(dtype)
        self.bg = w[f"{a}.to_gates.bias"].astype(dtype)
        self.wo = w[f"{a}.to_out.0.weight"].astype(np.float64).T.astype(dtype)   # [inner, dim]
        self.freqs = w[f"{a}.rotary_embed.freqs"].astype(np.float32)
        f = f"{p}.layers.0.1.net"
        fnorm = w[f"{f}.0.gamma"].astype(np.float64) * root
        self.w1 = (w[f"{f}.1.weight"].astype(np.float64) * fnorm[None, :]).T.astype(dtype)
        self.b1 = w[f"{f}.1.bias"].astype(dtype)
        self.w2 = w[f"{f}.4.weight"].astype(np.float64).T.astype(dtype)
        self.b2 = w[f"{f}.4.bias"].astype(dtype)
        self.out_scale = (w[f"{p}.norm.gamma"].astype(np.float64) * root).astype(dtype) \
            if normalized else None
        self.heads, self.hd, self.dtype = heads, hd, dtype
        if wround is not None:  # precision study: the folded weights as a 16-bit kernel holds them
            for name in ("wq", "wk", "wv", "wg", "wo", "w1", "w2"):
                setattr(self, name, wround(getattr(self, name)).astype(dtype))

    def attention(self, x: np.ndarray, tokens_cos_sin) -> np.ndarray:
        """Gated attention block output before the residual (roformer.rs:258-270)."""
        (qc, qs), (kc, ks) = tokens_cos_sin
        g, n, _ = x.shape
        h, d = self.heads, self.hd
        xn = unit_norm(x)
        q = rope_apply(xn @ self.wq, qc, qs, h).reshape(g, n, h, d)
        k = rope_apply(xn @ self.wk, kc, ks, h).reshape(g, n, h, d)
        v = (xn @ self.wv).reshape(g, n, h, d)
        out = np.empty((g, n, h, d), dtype=self.dtype)
        qh = q.transpose(0, 2, 1, 3)                      # [g, h, n, d], q carries 1/sqrt(d)
        kt = k.transpose(0, 2, 3, 1)                      # [g, h, d, n]
        vh = v.transpose(0, 2, 1, 3)                      # [g, h, n, d]
        step = max(1, int(2e7 // max(1, h * n * n)))  # bound the score tensor
        for g0 in range(0, g, step):
            sl = slice(g0, g0 + step)
            s = np.matmul(qh[sl], kt[sl])
            s -= s.max(axis=3, keepdims=True)
            e = np.exp(s)
            e /= e.sum(axis=3, keepdims=True)
            out[sl] = np.matmul(e, vh[sl]).transpose(0, 2, 1, 3)
        gates = sigmoid(xn @ self.wg + self.bg)
        out = out * gates[..., None]
        return out.reshape(g, n, h * d) @ self.wo

    def forward(self, x: np.ndarray, rope) -> np.ndarray:
        x = self.attention(x, rope) + x
        hidden = gelu(unit_norm(x) @ self.w1 + self.b1)
        y = hidden @ self.w2 + self.b2 + x
        if self.out_scale is not None:
            y = unit_norm(y) * self.out_scale
        return y


class Roformer:
    """Band split → ``depth`` × (time, band) transformers → mask heads (network.rs:59-400).

    ``weight_round`` (precision studies only) maps every transformer and mask-head weight matrix,
    after load-time folding, through a rounding function, e.g. to bf16 or f16 values: the error
    of that model bounds what any kernel holding those weights in that format can reach.
    """

    def __init__(self, package: str, dtype=np.float64, weight_round=None):
        with open(os.path.join(package, "manifest.json")) as fh:
            self.manifest = json.load(fh)
        c = self.manifest["config"]
        self.config, self.dtype = c, dtype
        w = load_file(os.path.join(package, "model.safetensors"))
        self._used = set()
        wt = _Tracker(w, self._used)
        dim, nb = c["dim"], len(c["bands"])
        self.bands = [list(b) for b in c["bands"]]
        self.split = []
        for band, bins in enumerate(self.bands):
            width = len(bins) * 4
            p = f"band_split.to_features.{band}"
            scale = wt[f"{p}.0.gamma"].astype(np.float64) * math.sqrt(width)
            W = wt[f"{p}.1.weight"].astype(np.float64) * scale[None, :]     # [dim, width]
            self.split.append((W.T.astype(dtype), wt[f"{p}.1.bias"].astype(dtype)))
        normalized = c["family"] == "mel-band-roformer"
        self.normalized = normalized
        self.axes = [(Transformer(wt, f"layers.{i}.0", c, normalized, dtype, weight_round),
                      Transformer(wt, f"layers.{i}.1", c, normalized, dtype, weight_round))
                     for i in range(c["depth"])]
        self.final_norm = None if normalized else \
            (wt["final_norm.gamma"].astype(np.float64) * math.sqrt(dim)).astype(dtype)
        hidden_layers = c["mask_depth"] if normalized else c["mask_depth"] - 1
        self.masks = []
        for stem in range(len(c["stems"])):
            heads = []
            for band, bins in enumerate(self.bands):
                key = lambda layer: f"mask_estimators.{stem}.to_freqs.{band}.0.{layer * 2}"
                hid = [(wt[f"{key(l)}.weight"].astype(dtype).T, wt[f"{key(l)}.bias"].astype(dtype))
                       for l in range(hidden_layers)]
                width = len(bins) * 4
                W = wt[f"{key(hidden_layers)}.weight"].astype(dtype)          # [2·width, in]
                b = wt[f"{key(hidden_layers)}.bias"].astype(dtype)
                wv, wg = W[:width].T, W[width:].T
                if weight_round is not None:
                    hid = [(weight_round(h).astype(dtype), bh) for h, bh in hid]
                    wv, wg = weight_round(wv).astype(dtype), weight_round(wg).astype(dtype)
                heads.append((hid, wv, b[:width], wg, b[width:]))
            self.masks.append(heads)
        unused = set(w) - self._used
        if unused:
            raise ValueError(f"unrecognized checkpoint tensors: {sorted(unused)[:8]}")
        bins = c["n_fft"] // 2 + 1
        self.coverage = np.zeros(2 * bins)
        for b in self.bands:
            for f in b:
                self.coverage[2 * f] += 1
                self.coverage[2 * f + 1] += 1

    def forward(self, spectrum: np.ndarray) -> np.ndarray:
        """``[frames, rows·2]`` → masks ``[stems, rows, 2, frames]`` (network.rs:303-400)."""
        c = self.config
        t, columns = spectrum.shape
        bins = c["n_fft"] // 2 + 1
        rows = bins * 2
        if t == 0 or columns != rows * 2:
            raise ValueError("invalid model spectrum shape")
        spec = spectrum.astype(self.dtype)
        nb = len(self.bands)
        x = np.empty((nb, t, c["dim"]), dtype=self.dtype)
        for band, bins_b in enumerate(self.bands):
            cols = (4 * np.asarray(bins_b)[:, None] + np.arange(4)[None, :]).ravel()
            W, b = self.split[band]
            x[band] = unit_norm(spec[:, cols]) @ W + b
        time_rope = self._rope(t)
        band_rope = self._rope(nb)
        for time, freq in self.axes:
            x = time.forward(x, time_rope(time.freqs))
            y = np.ascontiguousarray(x.transpose(1, 0, 2))
            x = np.ascontiguousarray(freq.forward(y, band_rope(freq.freqs)).transpose(1, 0, 2))
        if self.final_norm is not None:
            x = unit_norm(x) * self.final_norm
        out = np.zeros((len(self.masks), rows, 2, t), dtype=self.dtype)
        for s, heads in enumerate(self.masks):
            acc = np.zeros((rows, 2, t), dtype=self.dtype)
            for band, bins_b in enumerate(self.bands):
                hid, wv, bv, wg, bg = heads[band]
                h = x[band]
                for W, b in hid:
                    h = np.tanh(h @ W + b)
                m = (h @ wv + bv) * sigmoid(h @ wg + bg)              # [t, width]
                m = m.T.reshape(len(bins_b) * 2, 2, t)                 # rows (bin, ch), re/im
                target = (2 * np.asarray(bins_b)[:, None] + np.arange(2)[None, :]).ravel()
                acc[target] += m
            out[s] = acc / self.coverage[:, None, None]
        return out

    def _rope(self, tokens: int):
        d = self.config["head_dim"]
        cache = {}

        def get(freqs):
            key = freqs.tobytes()
            if key not in cache:
                cache[key] = (rope_tables(freqs, tokens, 1.0 / math.sqrt(d)),
                              rope_tables(freqs, tokens, 1.0))
            return cache[key]
        return get


class _Tracker(dict):
    """Mapping that records which tensors were read (the strict loader of weights.rs:130-144)."""

    def __init__(self, w, used):
        super().__init__(w)
        self._used = used

    def __getitem__(self, key):
        self._used.add(key)
        return super().__getitem__(key)
