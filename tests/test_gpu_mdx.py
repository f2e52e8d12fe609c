"""Classic MDX ONNX graphs on the GPU through the C ABI: the reference's graph known answers
(crates/ancha-models/tests/mdx_contracts.rs) and a synthetic TFC-TDF-style graph against the
numpy oracle (oracle/mdx.py), in f32."""
import ctypes as C

import numpy as np
import pytest

from ancha_b200 import _native as N
from ancha_b200.onnx_writer import Attr, Node, model
from oracle import mdx as M

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def run(torch, onnx, x, optimized=True):
    from ancha_b200.mdx import Graph
    g = Graph(onnx, 0, optimized, gemm=None)  # the direct kernels (conv_gemm: test_gpu_mdx_gemm.py)
    return g.forward(torch.from_numpy(np.asarray(x, np.float32)).cuda()).cpu().numpy().astype(np.float64)


def test_known_answer_graphs(torch_cuda):
    import test_oracle_mdx as T  # the graphs of the oracle tests
    x = np.array([1.0, -2.0, 0.0, 4.0]).reshape(1, 1, 2, 2)
    for optimized in (False, True):
        y = run(torch_cuda, T.fold_graph(), x, optimized)
        for c in range(2):
            for i, v in enumerate([1.0, -2.0, 0.0, 4.0]):
                e = max(((v * [2.0, -1.0][c] + [0.25, -0.75][c]) - [0.8, -1.2][c])
                        / np.sqrt([0.5, 2.0][c] + 1e-5) * [1.5, 0.5][c] + [0.4, -0.3][c], 0.0)
                assert abs(y.ravel()[c * 4 + i] - e) < 2e-6
    assert run(torch_cuda, T.chain_graph(), [[[[1.0, 2.0], [3.0, 4.0]]]]).ravel().tolist() == [8, 18, 12, 26]
    batched = np.arange(1.0, 9.0).reshape(2, 1, 2, 2)
    assert run(torch_cuda, T.chain_graph(), batched).ravel().tolist() == [8, 18, 12, 26, 28, 38, 40, 54]


def tfc_tdf_graph(f=64, t=32, seed=0):
    """Conv + BN + ReLU stacks (one grouped and dilated), a TDF pair over frequency through
    Transpose / MatMul, a strided down-convolution, a transposed up-convolution whose BN folds,
    skip additions, a per-channel Mul and a final strided ConvTranspose with output padding."""
    rng = np.random.default_rng(seed)
    w = {}

    def p(name, *shape, scale=None):
        fan = int(np.prod(shape[1:])) if len(shape) > 1 else 1
        w[name] = rng.standard_normal(shape) * (scale if scale is not None else 1.0 / np.sqrt(fan))
        return name

    def bn(prefix, c):
        w[prefix + "_g"] = 1.0 + 0.1 * rng.standard_normal(c)
        w[prefix + "_b"] = 0.1 * rng.standard_normal(c)
        w[prefix + "_m"] = 0.1 * rng.standard_normal(c)
        w[prefix + "_v"] = 0.5 + rng.random(c)
        return [prefix + s for s in ("_g", "_b", "_m", "_v")]

    n = []
    n += [Node("Conv", ["x", p("c1w", 8, 4, 3, 3), p("c1b", 8, scale=0.1)], "c1",
               attrs=[Attr("pads", ints=[1, 1, 1, 1]), Attr("kernel_shape", ints=[3, 3])]),
          Node("BatchNormalization", ["c1"] + bn("bn1", 8), "b1", attrs=[Attr("epsilon", f=1e-5)]),
          Node("Relu", ["b1"], "r1"),
          Node("Conv", ["r1", p("c2w", 8, 4, 3, 3), p("c2b", 8, scale=0.1)], "c2",
               attrs=[Attr("pads", ints=[2, 2, 2, 2]), Attr("dilations", ints=[2, 2]), Attr("group", i=2)]),
          Node("BatchNormalization", ["c2"] + bn("bn2", 8), "b2"),
          Node("Relu", ["b2"], "r2"),
          Node("Transpose", ["r2"], "tr", attrs=[Attr("perm", ints=[0, 1, 3, 2])]),
          Node("MatMul", ["tr", p("tdf1", f, f // 4)], "m1"),
          Node("Relu", ["m1"], "mr"),
          Node("MatMul", ["mr", p("tdf2", f // 4, f)], "m2"),
          Node("Transpose", ["m2"], "tb", attrs=[Attr("perm", ints=[0, 1, 3, 2])]),
          Node("Add", ["tb", "r2"], "s1"),
          Node("Conv", ["s1", p("dw", 16, 8, 2, 2), p("db", 16, scale=0.1)], "d1", attrs=[Attr("strides", ints=[2, 2])]),
          Node("BatchNormalization", ["d1"] + bn("bn3", 16), "b3"),
          Node("Relu", ["b3"], "r3"),
          Node("ConvTranspose", ["r3", p("uw", 16, 8, 2, 2), p("ub", 8, scale=0.1)], "u1",
               attrs=[Attr("strides", ints=[2, 2])]),
          Node("BatchNormalization", ["u1"] + bn("bn4", 8), "b4"),
          Node("Relu", ["b4"], "r4"),
          Node("Add", ["r4", "s1"], "s2"),
          Node("Conv", ["s2", p("pw", 8, 8, 1, 1)], "c3"),
          Node("Mul", ["c3", p("scale", 1, 8, 1, 1, scale=1.0)], "c4"),
          Node("ConvTranspose", ["c4", p("ow", 8, 4, 3, 3), p("ob", 4, scale=0.1)], "out",
               attrs=[Attr("strides", ints=[2, 2]), Attr("pads", ints=[1, 1, 1, 1]),
                      Attr("output_padding", ints=[1, 1])])]
    return model(n, w), w


@pytest.mark.parametrize("optimized", [False, True])
@pytest.mark.parametrize("batch", [1, 2])
def test_synthetic_graph_matches_oracle(torch_cuda, optimized, batch):
    onnx, _ = tfc_tdf_graph()
    ref_graph = M.Graph(onnx, optimized)
    x = np.random.default_rng(3).standard_normal((batch, 4, 64, 32))
    ref = ref_graph.forward(x)
    y = run(torch_cuda, onnx, x, optimized)
    assert y.shape == ref.shape == (batch, 4, 128, 64)
    err = np.abs(y - ref).max() / np.abs(ref).max()
    print(f"classic MDX graph batch {batch} optimized={optimized}: max |d| / max |ref| {err:.2e}")
    assert err < 1e-5
    if optimized:
        assert ref_graph.folded_bn == 1  # the BN after the up-convolution


def test_shape_errors_and_cancellation(torch_cuda):
    from ancha_b200.mdx import Graph
    onnx, _ = tfc_tdf_graph()
    g = Graph(onnx)
    with pytest.raises(N.AnchaError) as e:
        g.output_shape((1, 3, 64, 32))  # 3 input channels against a 4-channel convolution
    assert e.value.status == N.E_INVALID
    with pytest.raises(N.AnchaError) as e:
        g.forward(torch_cuda.zeros((1, 4, 64, 32), device="cuda"), cancel=C.c_int(1))
    assert e.value.status == N.E_CANCELLED
    assert g.output_shape((2, 4, 64, 32)) == (2, 4, 128, 64)


def shape_preserving_graph(seed=1):
    rng = np.random.default_rng(seed)
    w = {"c1w": rng.standard_normal((8, 4, 3, 3)) / 6.0, "c1b": 0.1 * rng.standard_normal(8),
         "g": 1.0 + 0.1 * rng.standard_normal(8), "b": 0.1 * rng.standard_normal(8),
         "m": 0.1 * rng.standard_normal(8), "v": 0.5 + rng.random(8),
         "c2w": rng.standard_normal((4, 8, 1, 1)) / 3.0}
    n = [Node("Conv", ["x", "c1w", "c1b"], "c1", attrs=[Attr("pads", ints=[1, 1, 1, 1])]),
         Node("BatchNormalization", ["c1", "g", "b", "m", "v"], "bn"), Node("Relu", ["bn"], "r"),
         Node("Conv", ["r", "c2w"], "out")]
    return model(n, w)


@pytest.mark.parametrize("n_fft,hop,bins,opts", [
    (512, 128, 256, dict(batch=1)),                      # n_fft / 2 = 2^8
    (384, 96, 160, dict(batch=3, overlap=0.5)),         # 3 · 2^6: radix-3 combination
    (320, 80, 128, dict(batch=2, overlap=0.0, denoise=True)),  # 5 · 2^5: radix-5, rectangular, denoise
])
def test_separate_task_matches_oracle(torch_cuda, n_fft, hop, bins, opts):
    from ancha_b200.mdx import Graph
    onnx = shape_preserving_graph()
    x = (np.random.default_rng(7).standard_normal((2, 4000)) * 0.1).astype(np.float32)
    ref_p, ref_r = M.separate(M.Graph(onnx, True), n_fft, bins, 16, 1.035, x.astype(np.float64), hop=hop, **opts)
    p, r, secs = Graph(onnx, gemm=None).separate_pcm(x, n_fft=n_fft, hop=hop, bins=bins, frames=16, compensate=1.035, **opts)
    err = np.abs(p - ref_p).max() / np.abs(ref_p).max()
    print(f"classic MDX task n_fft {n_fft} {opts}: max |d| / max |ref| {err:.2e}, {secs * 1e3:.1f} ms")
    assert err < 2e-5
    assert np.abs(p + r - x).max() < 1e-6


def test_separate_task_rejects_bad_options(torch_cuda):
    from ancha_b200.mdx import Graph
    g = Graph(shape_preserving_graph())
    x = np.zeros((2, 4000), np.float32)
    for bad in (dict(overlap=0.99), dict(batch=5), dict(n_fft=448),  # 448 / 2 = 7 · 2^5
                dict(overlap=float("nan")), dict(hop=1024),           # hop above n_fft
                dict(frames=1 << 20)):                                 # a chunk past 60 s
        with pytest.raises(N.AnchaError):
            g.separate_pcm(x, **dict(dict(n_fft=512, hop=128, bins=256, frames=16), **bad))
    with pytest.raises(N.AnchaError) as e:
        g.separate_pcm(x, n_fft=512, hop=128, bins=256, frames=16, cancel=C.c_int(1))
    assert e.value.status == N.E_CANCELLED
