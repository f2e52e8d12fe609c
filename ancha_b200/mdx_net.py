"""Synthetic classic MDX-Net graphs (TFC-TDF v1 U-Net) as ONNX: the classic MDX-Net benchmark
workload (n_fft 6144, tiles of 3072 bins × 256 frames).

The registered classic MDX checkpoints (crates/ancha-models/src/mdx.rs:36-93) are not available
here, so this module writes a graph of the same family with random weights: the TFC-TDF v1 U-Net
of the MDX-Net papers, in the form an eval-mode ONNX export takes and the classic MDX executor
reads (opset 13; ``mdx.rs:161-472``):

* input ``x`` [b, 4, F, T] (L.re, L.im, R.re, R.im of F bins × T frames), first a 1 × 1 Conv to
  ``g`` channels + Relu, then a Transpose to [b, c, T, F] so the TDF Linears act on frequency;
* ``scales`` encoder levels, each a TFC-TDF block followed by a 2 × 2 / stride-2 Conv to
  c + g channels + Relu; a middle TFC-TDF block; ``scales`` decoder levels, each a 2 × 2 /
  stride-2 ConvTranspose to c − g channels + BatchNormalization + Relu, a Mul with the encoder
  block output of the same level (the multiplicative skip) and a TFC-TDF block; a Transpose back
  and a final 1 × 1 Conv to 4 channels;
* TFC-TDF block on c channels and f frequencies: ``layers`` 3 × 3 Convs (c → c, padding 1) +
  Relu, then x + TDF(x) with TDF = MatMul [f, f / bottleneck] + BatchNormalization + Relu +
  MatMul [f / bottleneck, f] + BatchNormalization + Relu.

Convolutions carry a bias and no BatchNormalization of their own (an eval export folds Conv +
BatchNormalization into the Conv); ConvTranspose keeps its BatchNormalization, which the executor
folds when optimized. Weights are LeCun-uniform, U(±√(3 / fan_in)): with five scales,
He-uniform weights (twice the variance) let the residual adds and multiplicative skips grow the
output to ~1e8 for unit input, past the f16 range, while these keep it near 0.04 rms. Biases and
BatchNormalization statistics are small and seeded.
The channel growth ``g`` and the other widths of the real checkpoints are not known here; the
defaults are a stand-in of the same structure.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .onnx_writer import Attr, Node, model


@dataclass
class MdxNetConfig:
    dim_f: int = 3072      # frequency bins of a tile ("mdx-inst-hq-2")
    dim_t: int = 256       # frames of a tile
    channels: int = 4      # stereo complex input
    growth: int = 48       # channels added per encoder level (stand-in)
    scales: int = 5
    layers: int = 3        # 3 × 3 convolutions per TFC
    bottleneck: int = 8    # TDF hidden width f / bottleneck

    def validate(self) -> None:
        d = 1 << self.scales
        if self.dim_f % d or self.dim_t % d or (self.dim_f // d) % self.bottleneck or min(
                self.growth, self.layers, self.bottleneck, self.scales) < 1:
            raise ValueError("frequency and time must survive every 2 × 2 stride and the TDF bottleneck")


def tfc_tdf_v1(c: MdxNetConfig = MdxNetConfig(), seed: int = 0) -> bytes:
    """ONNX bytes of a random-weight TFC-TDF v1 U-Net with configuration ``c``."""
    c.validate()
    rng = np.random.default_rng(seed)
    nodes, weights = [], {}
    counter = [0]

    def name(prefix):
        counter[0] += 1
        return f"{prefix}{counter[0]}"

    def lecun(shape, fan_in):
        bound = np.sqrt(3.0 / fan_in)
        return rng.uniform(-bound, bound, shape).astype(np.float32)

    def bias(n, fan_in):
        return rng.uniform(-0.1, 0.1, n).astype(np.float32) / np.sqrt(fan_in)

    def conv(x, ci, co, k, stride=1, pad=0, transpose=False):
        w, b, y = name("w"), name("b"), name("v")
        if transpose:
            weights[w] = lecun((ci, co, k, k), ci)  # ConvTranspose weights [ci][co][kh][kw]
        else:
            weights[w] = lecun((co, ci, k, k), ci * k * k)
        weights[b] = bias(co, ci * k * k)
        attrs = [Attr("kernel_shape", ints=[k, k]), Attr("strides", ints=[stride, stride])]
        if pad:
            attrs.append(Attr("pads", ints=[pad] * 4))
        nodes.append(Node("ConvTranspose" if transpose else "Conv", [x, w, b], y, name=y, attrs=attrs))
        return y

    def batchnorm(x, ch):
        p = name("bn")
        weights[p + "_g"] = (1.0 + 0.05 * rng.standard_normal(ch)).astype(np.float32)
        weights[p + "_b"] = (0.05 * rng.standard_normal(ch)).astype(np.float32)
        weights[p + "_m"] = (0.05 * rng.standard_normal(ch)).astype(np.float32)
        weights[p + "_v"] = (1.0 + 0.1 * rng.random(ch)).astype(np.float32)
        y = name("v")
        nodes.append(Node("BatchNormalization", [x, p + "_g", p + "_b", p + "_m", p + "_v"], y, name=y,
                          attrs=[Attr("epsilon", f=1e-5)]))
        return y

    def op(kind, inputs, attrs=()):
        y = name("v")
        nodes.append(Node(kind, list(inputs), y, name=y, attrs=list(attrs)))
        return y

    def linear(x, fi, fo):
        w = name("w")
        weights[w] = lecun((fi, fo), fi)  # MatMul right operand [in, out]
        return op("MatMul", [x, w])

    def tfc_tdf(x, ch, f):
        for _ in range(c.layers):
            x = op("Relu", [conv(x, ch, ch, 3, pad=1)])
        t = op("Relu", [batchnorm(linear(x, f, f // c.bottleneck), ch)])
        t = op("Relu", [batchnorm(linear(t, f // c.bottleneck, f), ch)])
        return op("Add", [x, t])

    x = op("Relu", [conv("x", c.channels, c.growth, 1)])
    x = op("Transpose", [x], [Attr("perm", ints=[0, 1, 3, 2])])
    ch, f, skips = c.growth, c.dim_f, []
    for _ in range(c.scales):
        x = tfc_tdf(x, ch, f)
        skips.append(x)
        x = op("Relu", [conv(x, ch, ch + c.growth, 2, stride=2)])
        ch, f = ch + c.growth, f // 2
    x = tfc_tdf(x, ch, f)
    for i in range(c.scales):
        x = op("Relu", [batchnorm(conv(x, ch, ch - c.growth, 2, stride=2, transpose=True), ch - c.growth)])
        ch, f = ch - c.growth, f * 2
        x = op("Mul", [x, skips[-1 - i]])
        x = tfc_tdf(x, ch, f)
    x = op("Transpose", [x], [Attr("perm", ints=[0, 1, 3, 2])])
    conv(x, ch, c.channels, 1)
    nodes[-1].output = nodes[-1].name = "out"  # the graph output
    return model(nodes, weights, inputs=("x",), outputs=("out",))


def forward_flops(c: MdxNetConfig = MdxNetConfig(), batch: int = 1) -> float:
    """Multiply-adds × 2 of one forward over ``batch`` tiles (convolutions, transposed
    convolutions and TDF MatMuls; elementwise work excluded)."""
    c.validate()
    ch, f, t = c.growth, c.dim_f, c.dim_t

    def tfc_tdf(ch, f, t):
        pos = f * t
        return c.layers * 9 * ch * ch * pos + 2 * ch * t * f * (f // c.bottleneck)

    macs = c.channels * c.growth * c.dim_f * c.dim_t  # first 1 × 1
    for _ in range(c.scales):
        macs += tfc_tdf(ch, f, t)
        macs += 4 * ch * (ch + c.growth) * (f // 2) * (t // 2)  # 2 × 2 / 2 down
        ch, f, t = ch + c.growth, f // 2, t // 2
    macs += tfc_tdf(ch, f, t)
    for _ in range(c.scales):
        macs += 4 * ch * (ch - c.growth) * f * t  # 2 × 2 / 2 transposed, per input position
        ch, f, t = ch - c.growth, f * 2, t * 2
        macs += tfc_tdf(ch, f, t)
    macs += ch * c.channels * c.dim_f * c.dim_t  # final 1 × 1
    return 2.0 * macs * batch
