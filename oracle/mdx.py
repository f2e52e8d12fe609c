"""Classic MDX ONNX executor in numpy (test oracle only).

Restates ``crates/ancha-models/src/mdx.rs``: ``Graph::from_bytes`` (mdx.rs:161-472) — opset-13
check, one input and one output, FLOAT initializers of at most four dims (left-padded to four,
finite), the attribute allow-list, symmetric convolution pads, eval-mode BatchNormalization
and, when ``optimized``, folding a BatchNormalization into the ConvTranspose that is its only
producer (mdx.rs:216-294) — and ``Graph::forward`` (mdx.rs:474-568): Conv / ConvTranspose with
stride, padding, dilation, groups and output padding, Relu, Transpose, MatMul and Add / Mul
with numpy broadcasting over NCHW tensors, BatchNormalization as (x − mean)/√(var + ε)·γ + β
or its folded affine form. Arithmetic is float64.

The protobuf reader below is this oracle's own, independent of the library's C++ reader.
``pack`` / ``unpack`` / ``separate`` restate the task of ``src/mdx_runtime.rs:79-248`` (three
zeroed low bins, UVR trim and pad, Hann-weighted chunk overlap-add, compensation, denoise).
"""
from __future__ import annotations

import struct

import math
import numpy as np

OPS = {"Conv", "ConvTranspose", "Relu", "Transpose", "MatMul", "Add", "Mul", "BatchNormalization"}


class GraphError(ValueError):
    pass


def _fields(buf: bytes):
    """(field number, wire type, value) of one protobuf message; length-delimited values are
    bytes, varints ints, fixed32 / fixed64 raw bytes."""
    i, n = 0, len(buf)
    while i < n:
        key, i = _read_varint(buf, i)
        f, w = key >> 3, key & 7
        if w == 0:
            v, i = _read_varint(buf, i)
        elif w == 1:
            v, i = buf[i:i + 8], i + 8
        elif w == 2:
            ln, i = _read_varint(buf, i)
            v, i = buf[i:i + ln], i + ln
        elif w == 5:
            v, i = buf[i:i + 4], i + 4
        else:
            raise GraphError(f"unsupported protobuf wire type {w}")
        if i > n:
            raise GraphError("truncated protobuf message")
        yield f, w, v


def _read_varint(buf: bytes, i: int):
    v, shift = 0, 0
    while True:
        if i >= len(buf):
            raise GraphError("truncated varint")
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        if not b & 0x80:
            return v, i
        shift += 7


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= 1 << 63 else v


def _ints(w, v):
    if w == 2:  # packed
        out, i = [], 0
        while i < len(v):
            x, i = _read_varint(v, i)
            out.append(_signed(x))
        return out
    return [_signed(v)]


def _attribute(buf):
    a = {"name": "", "type": 0, "ints": [], "i": None, "f": None}
    for f, w, v in _fields(buf):
        if f == 1:
            a["name"] = v.decode()
        elif f == 20:
            a["type"] = v
        elif f == 3:
            a["i"] = _signed(v)
        elif f == 2:
            a["f"] = struct.unpack("<f", v)[0]
        elif f == 8:
            a["ints"] += _ints(w, v)
    return a


def _node(buf):
    n = {"inputs": [], "outputs": [], "name": "", "op_type": "", "domain": "", "attrs": {}}
    for f, w, v in _fields(buf):
        if f == 1:
            n["inputs"].append(v.decode())
        elif f == 2:
            n["outputs"].append(v.decode())
        elif f == 3:
            n["name"] = v.decode()
        elif f == 4:
            n["op_type"] = v.decode()
        elif f == 7:
            n["domain"] = v.decode()
        elif f == 5:
            a = _attribute(v)
            n["attrs"][a["name"]] = a
    return n


def _tensor(buf):
    t = {"dims": [], "data_type": 0, "name": "", "raw": None, "floats": [], "external": False}
    for f, w, v in _fields(buf):
        if f == 1:
            t["dims"] += _ints(w, v)
        elif f == 2:
            t["data_type"] = v
        elif f == 8:
            t["name"] = v.decode()
        elif f == 9:
            t["raw"] = v
        elif f == 4:
            t["floats"] += list(np.frombuffer(v, "<f4")) if w == 2 else [struct.unpack("<f", v)[0]]
        elif f == 14 and v == 1:
            t["external"] = True
    return t


def _value_name(buf):
    for f, _, v in _fields(buf):
        if f == 1:
            return v.decode()
    return ""


def parse(model_bytes: bytes) -> dict:
    """The ModelProto subset of the executor: opset imports and the graph."""
    m = {"opset": [], "graph": None}
    for f, _, v in _fields(model_bytes):
        if f == 8:
            d = {"domain": "", "version": 0}
            for ff, _, vv in _fields(v):
                if ff == 1:
                    d["domain"] = vv.decode()
                elif ff == 2:
                    d["version"] = _signed(vv)
            m["opset"].append(d)
        elif f == 7:
            g = {"nodes": [], "initializers": [], "sparse": 0, "inputs": [], "outputs": []}
            for ff, _, vv in _fields(v):
                if ff == 1:
                    g["nodes"].append(_node(vv))
                elif ff == 5:
                    g["initializers"].append(_tensor(vv))
                elif ff == 15:
                    g["sparse"] += 1
                elif ff == 11:
                    g["inputs"].append(_value_name(vv))
                elif ff == 12:
                    g["outputs"].append(_value_name(vv))
            m["graph"] = g
    return m


def _int_attr(n, key, default):
    a = n["attrs"].get(key)
    return default if a is None or a["i"] is None else a["i"]


def _ints_attr(n, key, default):
    a = n["attrs"].get(key)
    return list(default) if a is None else list(a["ints"])


def _float_attr(n, key, default):
    a = n["attrs"].get(key)
    return default if a is None or a["f"] is None else a["f"]


def _pair(v, positive):
    if len(v) != 2 or any(x < (1 if positive else 0) for x in v):
        raise GraphError("invalid pair attribute")
    return int(v[0]), int(v[1])


ALLOWED = {"Conv": {"dilations", "group", "kernel_shape", "pads", "strides", "output_padding"},
           "ConvTranspose": {"dilations", "group", "kernel_shape", "pads", "strides", "output_padding"},
           "BatchNormalization": {"epsilon", "momentum", "training_mode"}, "Transpose": {"perm"}}


class Graph:
    """``Graph::from_bytes`` + ``Graph::forward`` (mdx.rs:161-568)."""

    def __init__(self, model_bytes: bytes, optimized: bool = True):
        m = parse(model_bytes)
        if len(m["opset"]) != 1 or m["opset"][0]["domain"] != "" or m["opset"][0]["version"] != 13:
            raise GraphError("classic MDX executor requires ONNX opset 13")
        g = m["graph"]
        if g is None:
            raise GraphError("missing ONNX graph")
        if len(g["inputs"]) != 1 or len(g["outputs"]) != 1 or g["sparse"]:
            raise GraphError("expected one input and one output, no sparse initializers")
        raw = {}
        for t in g["initializers"]:
            dims = t["dims"]
            if t["data_type"] != 1 or len(dims) > 4 or any(d <= 0 for d in dims) or t["external"]:
                raise GraphError(f"unsupported initializer {t['name']}")
            data = np.frombuffer(t["raw"], "<f4") if t["raw"] is not None else np.array(t["floats"], "<f4")
            shape = [1] * (4 - len(dims)) + list(dims)
            if data.size != math.prod(shape) or not np.all(np.isfinite(data)):  # exact, no int64 wrap
                raise GraphError(f"invalid initializer {t['name']}")
            if t["name"] in raw:
                raise GraphError("duplicate initializer")
            raw[t["name"]] = data.astype(np.float64).reshape(shape)
        nodes = g["nodes"]
        consumers = {}
        for n in nodes:
            for s in n["inputs"]:
                consumers[s] = consumers.get(s, 0) + 1
        skipped, redirected = set(), {}
        self.folded_bn = 0
        if optimized:
            for i, n in enumerate(nodes):
                if (n["op_type"] != "ConvTranspose" or len(n["outputs"]) != 1
                        or consumers.get(n["outputs"][0]) != 1 or g["outputs"][0] == n["outputs"][0]):
                    continue
                found = [(j, v) for j, v in enumerate(nodes)
                         if v["op_type"] == "BatchNormalization" and v["inputs"][:1] == n["outputs"][:1]]
                if not found:
                    continue
                j, bn = found[0]
                if len(bn["inputs"]) != 5 or len(bn["outputs"]) != 1 or _int_attr(bn, "training_mode", 0) != 0:
                    raise GraphError("unsupported BN")
                if len(n["inputs"]) != 3 or _int_attr(n, "group", 1) != 1:
                    raise GraphError("folding expects ungrouped transposed convolution with bias")
                gamma, beta, mean, var = (raw[bn["inputs"][k]].ravel() for k in range(1, 5))
                if not (len(gamma) == len(beta) == len(mean) == len(var)) or np.any(var < 0):
                    raise GraphError("invalid BN statistics")
                eps = _float_attr(bn, "epsilon", 1e-5)
                if not (eps > 0 and np.isfinite(eps)):
                    raise GraphError("invalid BN epsilon")
                scale = gamma / np.sqrt(var + eps)
                shift = beta - mean * scale
                w = raw[n["inputs"][1]]
                if w.shape[1] != len(scale):
                    raise GraphError("BN / ConvTranspose channel mismatch")
                bias = raw[n["inputs"][2]].ravel()
                if len(bias) != len(scale):
                    raise GraphError("invalid transpose bias")
                raw[f"__ancha_fold_{i}_weight"] = w * scale.reshape(1, -1, 1, 1)
                raw[f"__ancha_fold_{i}_bias"] = (bias * scale + shift).reshape(1, 1, 1, -1)
                skipped.add(j)
                redirected[i] = bn["outputs"][0]
                self.folded_bn += 1
        self.constants = dict(raw)
        self.input = g["inputs"][0]
        self.instructions = []
        seen = set(raw) | {self.input}
        for i, n in enumerate(nodes):
            if i in skipped:
                continue
            if n["domain"] or len(n["outputs"]) != 1:
                raise GraphError("unsupported node domain or multi-output")
            op = n["op_type"]
            if op not in OPS:
                raise GraphError(f"unsupported ONNX operation {op}")
            if any(a not in ALLOWED.get(op, set()) for a in n["attrs"]):
                raise GraphError(f"unsupported attribute in {n['name']}")
            inputs = list(n["inputs"])
            for s in inputs:
                if s not in seen:
                    raise GraphError(f"unknown input {s}")
            ins = {"op": op, "inputs": inputs}
            if op in ("Conv", "ConvTranspose"):
                if len(inputs) not in (2, 3):
                    raise GraphError("invalid conv inputs")
                pads = _ints_attr(n, "pads", [0, 0, 0, 0])
                if len(pads) != 4 or pads[0] != pads[2] or pads[1] != pads[3]:
                    raise GraphError("asymmetric convolution unsupported")
                groups = _int_attr(n, "group", 1)
                if groups <= 0:
                    raise GraphError("invalid groups")
                if i in redirected:
                    inputs[1], inputs[2] = f"__ancha_fold_{i}_weight", f"__ancha_fold_{i}_bias"
                ins.update(stride=_pair(_ints_attr(n, "strides", [1, 1]), True),
                           padding=_pair(pads[:2], False),
                           dilation=_pair(_ints_attr(n, "dilations", [1, 1]), True), groups=groups,
                           padding_out=_pair(_ints_attr(n, "output_padding", [0, 0]), False))
            elif op in ("Relu", "Transpose"):
                if len(inputs) != 1:
                    raise GraphError(f"invalid {op} inputs")
                if op == "Transpose":
                    p = _ints_attr(n, "perm", [3, 2, 1, 0])
                    if len(p) != 4 or set(p) != {0, 1, 2, 3}:
                        raise GraphError("invalid permutation")
                    ins["perm"] = tuple(int(v) for v in p)
            elif op in ("MatMul", "Add", "Mul"):
                if len(inputs) != 2:
                    raise GraphError("invalid binary inputs")
            else:  # BatchNormalization
                if len(inputs) != 5 or _int_attr(n, "training_mode", 0) != 0:
                    raise GraphError("only eval BN supported")
                eps = _float_attr(n, "epsilon", 1e-5)
                if not (np.isfinite(eps) and eps > 0):
                    raise GraphError("invalid BN epsilon")
                gamma, beta, mean, var = (raw[inputs[k]].ravel() for k in range(1, 5))
                if not (len(gamma) == len(beta) == len(mean) == len(var)) or np.any(var < 0):
                    raise GraphError("invalid BN statistics")
                ins["eps"] = eps
                if optimized:
                    scale = gamma / np.sqrt(var + eps)
                    ins["affine"] = (scale.reshape(1, -1, 1, 1), (beta - mean * scale).reshape(1, -1, 1, 1))
            out = redirected.get(i, n["outputs"][0])
            if out in seen:
                raise GraphError("duplicate ONNX value")
            seen.add(out)
            ins["inputs"] = inputs
            ins["output"] = out
            self.instructions.append(ins)
        self.output = g["outputs"][0]
        if self.output not in seen:
            raise GraphError("graph output missing")
        self.nodes = len(nodes)

    def forward(self, x: np.ndarray, cancelled: bool = False) -> np.ndarray:
        values = dict(self.constants)
        values[self.input] = np.asarray(x, np.float64)
        for ins in self.instructions:
            if cancelled:
                raise GraphError("task cancelled")
            v = [values[s] for s in ins["inputs"]]
            op = ins["op"]
            if op == "Conv":
                y = conv2d(v[0], v[1], ins["stride"], ins["padding"], ins["dilation"], ins["groups"])
            elif op == "ConvTranspose":
                y = conv_transpose2d(v[0], v[1], ins["stride"], ins["padding"], ins["padding_out"],
                                     ins["dilation"], ins["groups"])
            if op in ("Conv", "ConvTranspose"):
                if len(v) == 3:
                    y = y + v[2].ravel().reshape(1, -1, 1, 1)
            elif op == "Relu":
                y = np.maximum(v[0], 0.0)
            elif op == "Transpose":
                y = np.transpose(v[0], ins["perm"])
            elif op == "MatMul":
                y = np.matmul(v[0], v[1])
            elif op == "Add":
                y = v[0] + v[1]
            elif op == "Mul":
                y = v[0] * v[1]
            elif op == "BatchNormalization":
                if "affine" in ins:
                    y = v[0] * ins["affine"][0] + ins["affine"][1]
                else:
                    c = lambda t: t.ravel().reshape(1, -1, 1, 1)
                    y = (v[0] - c(v[3])) / np.sqrt(c(v[4]) + ins["eps"]) * c(v[1]) + c(v[2])
            values[ins["output"]] = y
        return values[self.output]


def conv2d(x, w, stride, padding, dilation, groups):
    """PyTorch / Burn conv2d, weights [out, in / groups, kh, kw], no bias."""
    b, ci, h, wd = x.shape
    co, cig, kh, kw = w.shape
    if ci != cig * groups or co % groups:
        raise GraphError("conv2d channel mismatch")
    (sh, sw), (ph, pw), (dh, dw) = stride, padding, dilation
    oh = (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1
    ow = (wd + 2 * pw - dw * (kw - 1) - 1) // sw + 1
    xp = np.pad(x, ((0, 0), (0, 0), (ph, ph), (pw, pw)))
    out = np.zeros((b, co, oh, ow))
    cog = co // groups
    for g in range(groups):
        xs = xp[:, g * cig:(g + 1) * cig]
        ws = w[g * cog:(g + 1) * cog]
        for ky in range(kh):
            for kx in range(kw):
                patch = xs[:, :, ky * dh:ky * dh + sh * (oh - 1) + 1:sh, kx * dw:kx * dw + sw * (ow - 1) + 1:sw]
                out[:, g * cog:(g + 1) * cog] += np.einsum("bchw,oc->bohw", patch, ws[:, :, ky, kx])
    return out


def conv_transpose2d(x, w, stride, padding, padding_out, dilation, groups):
    """PyTorch / Burn conv_transpose2d, weights [in, out / groups, kh, kw], no bias: input
    position (i, j) and tap (ky, kx) add into output (i·s + ky·d − p, j·s + kx·d − p)."""
    b, ci, h, wd = x.shape
    wi, cog, kh, kw = w.shape
    if wi != ci or ci % groups:
        raise GraphError("conv_transpose channel mismatch")
    (sh, sw), (ph, pw), (oph, opw), (dh, dw) = stride, padding, padding_out, dilation
    oh = (h - 1) * sh - 2 * ph + dh * (kh - 1) + oph + 1
    ow = (wd - 1) * sw - 2 * pw + dw * (kw - 1) + opw + 1
    full = np.zeros((b, cog * groups, (h - 1) * sh + dh * (kh - 1) + 1 + oph, (wd - 1) * sw + dw * (kw - 1) + 1 + opw))
    cig = ci // groups
    for g in range(groups):
        xs = x[:, g * cig:(g + 1) * cig]
        for ky in range(kh):
            for kx in range(kw):
                contrib = np.einsum("bchw,co->bohw", xs, w[g * cig:(g + 1) * cig, :, ky, kx])
                full[:, g * cog:(g + 1) * cog, ky * dh:ky * dh + sh * (h - 1) + 1:sh,
                     kx * dw:kx * dw + sw * (wd - 1) + 1:sw] += contrib
    return full[:, :, ph:ph + oh, pw:pw + ow]


# ---- Task: src/mdx_runtime.rs -----------------------------------------------------------------

def pack(stft, planes: np.ndarray, bins: int, zero_low_bins: int = 3) -> np.ndarray:
    """``mdx_runtime::pack`` = ``spectral::pack`` with the lowest three bins zeroed
    (src/mdx_runtime.rs:79-83, src/spectral.rs:5-36): ``[2, n]`` → ``[4, bins, frames]``."""
    frames = planes.shape[1] // stft.hop + 1
    out = np.empty((4, bins, frames))
    for ch in range(2):
        spec = stft.forward(planes[ch])[:, :bins].copy()
        spec[:, :zero_low_bins] = 0.0
        out[2 * ch] = spec.real.T
        out[2 * ch + 1] = spec.imag.T
    return out


def unpack(stft, packed: np.ndarray, length: int) -> np.ndarray:
    """``spectral::unpack`` (src/spectral.rs:38-76): bins past ``bins`` are zero."""
    _, bins, frames = packed.shape
    out = []
    for ch in range(2):
        spec = np.zeros((frames, stft.n_fft // 2 + 1), dtype=np.complex128)
        spec[:, :bins] = packed[2 * ch].T + 1j * packed[2 * ch + 1].T
        out.append(stft.inverse(spec, length, False))
    return np.stack(out)


def separate(graph: Graph, n_fft: int, bins: int, frames: int, compensate: float, planes: np.ndarray,
             hop: int = 1024, overlap=None, denoise: bool = False, optimized: bool = True,
             batch: int = 1) -> tuple:
    """``separate_mdx`` without file I/O (src/mdx_runtime.rs:84-248): UVR trim / pad, chunks
    every ``gen_size`` samples (or (1 − overlap)·chunk), Hann-weighted overlap-add divided by
    the summed weights (rectangular for overlap 0), times ``compensate``; optional denoise
    (f(x) − f(−x))/2. Returns (predicted, residual), each ``[2, n]``."""
    from .dsp import Stft
    if not 1 <= batch <= 4:
        raise GraphError("MDX batch size must be between 1 and 4")
    if overlap is not None and not (np.isfinite(overlap) and 0.0 <= overlap <= 0.95):
        raise GraphError("MDX overlap must be between 0 and 0.95")
    n = planes.shape[1]
    chunk = hop * (frames - 1)
    trim = n_fft // 2
    gen_size = chunk - n_fft
    pad = gen_size + trim - n % gen_size
    mixture_len = trim + n + pad
    step = gen_size if overlap is None else int((1.0 - overlap) * chunk)
    if step <= 0:
        raise GraphError("zero MDX step")
    starts = [s for s in range(0, mixture_len, step) if not optimized or s < trim + n]
    stft = Stft(n_fft, hop)
    result = np.zeros((2, n))
    divisor = np.zeros(n)
    for b0 in range(0, len(starts), batch):
        group = starts[b0:b0 + batch]
        packed = []
        for s in group:
            actual = min(chunk, mixture_len - s)
            window = np.zeros((2, chunk))
            for i in range(actual):
                pos = s + i
                if trim <= pos < trim + n:
                    window[:, i] = planes[:, pos - trim]
            p = pack(stft, window, bins)
            if p.shape[2] != frames:
                raise GraphError("MDX frame mismatch")
            packed.append(p)
        x = np.stack(packed)
        y = (graph.forward(x) - graph.forward(-x)) * 0.5 if denoise else graph.forward(x)
        if y.shape != x.shape:
            raise GraphError("MDX output shape mismatch")
        for k, s in enumerate(group):
            audio = unpack(stft, y[k], chunk)
            actual = min(chunk, mixture_len - s)
            first, end = max(s, trim), min(s + actual, trim + n)
            for pos in range(first, end):
                local = pos - s
                w = 1.0 if overlap == 0.0 else float(np.float32(0.5 - 0.5 * np.cos(2 * np.pi * local / (actual - 1))))
                divisor[pos - trim] += w
                result[:, pos - trim] += audio[:, local] * w
    if np.any(divisor <= 0):
        raise GraphError("MDX OLA uncovered sample; overlap setting is invalid")
    predicted = result / divisor * compensate
    return predicted, planes - predicted
