"""A float64 PyTorch re-expression of the Mel-Band / BS-RoFormer forward (test helper).

It restates the reference's generic path from the PyTorch-style modules the checkpoint keys
name, independently of ``oracle/roformer.py``: nothing is folded at load time (every norm is
applied as ``x / max(‖x‖, 1e-12) · √d · γ`` before its Linear, where the oracle and the engine
fold ``√d · γ`` into the weights), attention is ``torch.nn.functional.scaled_dot_product_attention``,
RoPE multiplies interleaved pairs as complex numbers, GELU is ``torch.nn.functional.gelu``
(erf), the band split gathers with ``index_select`` and the mask heads scatter with
``index_add_``. Reference: crates/ancha-models/src/network.rs:89-400 (band split, axial loop,
final norm, mask heads, coverage), roformer.rs:16-55 (unit_norm, SourceNorm), roformer.rs:150-187
and 274-309 (RoPE: angle t·f in f32, the query side scaled by 1/√head_dim), roformer.rs:205-270
and 381-459 (attention with sigmoid gates, feed-forward, residuals).
"""
from __future__ import annotations

import json
import math
import os

import torch
import torch.nn.functional as F
from safetensors.torch import load_file


def _rms(x, gamma):
    """``x / max(‖x‖₂, 1e-12) · √d · γ`` over the last axis."""
    return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12) * math.sqrt(x.shape[-1]) * gamma


def _rope(x, freqs, heads):
    """Interleaved-pair rotary embedding of ``x [groups, tokens, heads·d]`` as a complex product."""
    g, n, w = x.shape
    t = torch.arange(n, dtype=torch.float32)[:, None]
    ang = (t * freqs.float()[None, :]).double()                       # [tokens, d/2], product in f32
    rot = torch.polar(torch.ones_like(ang), ang)                       # e^{i·angle}
    z = torch.view_as_complex(x.reshape(g, n, heads, -1, 2).contiguous())
    return torch.view_as_real(z * rot[None, :, None, :]).reshape(g, n, w)


class TorchRoformer:
    def __init__(self, package: str):
        with open(os.path.join(package, "manifest.json")) as fh:
            self.c = json.load(fh)["config"]
        self.w = {k: v.double() for k, v in load_file(os.path.join(package, "model.safetensors")).items()}

    def _transformer(self, x, p):
        c, w = self.c, self.w
        heads, hd = c["heads"], c["head_dim"]
        inner = heads * hd
        a, f = f"{p}.layers.0.0", f"{p}.layers.0.1.net"
        g, n, _ = x.shape
        xn = _rms(x, w[f"{a}.norm.gamma"])
        qkv = xn @ w[f"{a}.to_qkv.weight"].T
        q, k, v = qkv[..., :inner], qkv[..., inner:2 * inner], qkv[..., 2 * inner:]
        freqs = w[f"{a}.rotary_embed.freqs"]
        q = _rope(q, freqs, heads) / math.sqrt(hd)
        k = _rope(k, freqs, heads)
        split = lambda t: t.reshape(g, n, heads, hd).transpose(1, 2)   # [g, h, n, d]
        o = F.scaled_dot_product_attention(split(q), split(k), split(v), scale=1.0)
        gates = torch.sigmoid(xn @ w[f"{a}.to_gates.weight"].T + w[f"{a}.to_gates.bias"])  # [g, n, h]
        o = o.transpose(1, 2) * gates[..., None]                       # [g, n, h, d]
        x = x + o.reshape(g, n, inner) @ w[f"{a}.to_out.0.weight"].T
        h = F.gelu(_rms(x, w[f"{f}.0.gamma"]) @ w[f"{f}.1.weight"].T + w[f"{f}.1.bias"])
        y = h @ w[f"{f}.4.weight"].T + w[f"{f}.4.bias"] + x
        if self.c["family"] == "mel-band-roformer":
            y = _rms(y, w[f"{p}.norm.gamma"])
        return y

    def forward(self, spectrum) -> torch.Tensor:
        """``[frames, bins·4]`` → masks ``[stems, bins·2, 2, frames]``."""
        c, w = self.c, self.w
        spec = torch.as_tensor(spectrum).double()
        t = spec.shape[0]
        bands = [torch.tensor(b, dtype=torch.long) for b in c["bands"]]
        feats = []
        for i, bins in enumerate(bands):
            cols = (4 * bins[:, None] + torch.arange(4)[None, :]).reshape(-1)
            p = f"band_split.to_features.{i}"
            z = _rms(spec.index_select(1, cols), w[f"{p}.0.gamma"])
            feats.append(z @ w[f"{p}.1.weight"].T + w[f"{p}.1.bias"])
        x = torch.stack(feats)                                          # [bands, frames, dim]
        for layer in range(c["depth"]):
            x = self._transformer(x, f"layers.{layer}.0")               # time axis
            x = self._transformer(x.transpose(0, 1), f"layers.{layer}.1").transpose(0, 1)  # band axis
        mel = c["family"] == "mel-band-roformer"
        if not mel:
            x = _rms(x, w["final_norm.gamma"])
        rows = (c["n_fft"] // 2 + 1) * 2
        coverage = torch.zeros(rows, dtype=torch.float64)
        for bins in bands:
            coverage.index_add_(0, (2 * bins[:, None] + torch.arange(2)[None, :]).reshape(-1),
                                torch.ones(2 * len(bins), dtype=torch.float64))
        hidden = c["mask_depth"] if mel else c["mask_depth"] - 1
        out = []
        for s in range(len(c["stems"])):
            acc = torch.zeros(rows, 2, t, dtype=torch.float64)
            for i, bins in enumerate(bands):
                key = lambda l: f"mask_estimators.{s}.to_freqs.{i}.0.{2 * l}"
                h = x[i]
                for l in range(hidden):
                    h = torch.tanh(h @ w[f"{key(l)}.weight"].T + w[f"{key(l)}.bias"])
                glu = h @ w[f"{key(hidden)}.weight"].T + w[f"{key(hidden)}.bias"]
                m = F.glu(glu, dim=-1)                                   # value · σ(gate)
                m = m.T.reshape(len(bins) * 2, 2, t)
                acc.index_add_(0, (2 * bins[:, None] + torch.arange(2)[None, :]).reshape(-1), m)
            out.append(acc / coverage[:, None, None])
        return torch.stack(out)
