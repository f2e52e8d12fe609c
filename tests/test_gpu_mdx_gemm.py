"""Classic MDX graphs with conv_gemm (``ancha_mdx_set_gemm``; Graph::forward's option,
crates/ancha-models/src/mdx.rs:472-530): eligible convolutions as patch gather + GEMM and
constant-weight MatMuls as one GEMM, in f32 (FFMA) and with 16-bit operands on the tensor
cores, against the numpy oracle and against the direct kernels.
"""

import numpy as np
import pytest

from ancha_b200 import _native as N
from oracle import mdx as M

pytestmark = pytest.mark.gpu

# max |Δ| / max |ref| per mode: f32 as the direct kernels; 16-bit operands on every
# convolution of a ~10-layer graph. Rounding the operands of exactly the GEMM-run operations
# in numpy (f64 accumulation otherwise) gives 5.4e-4 (f16) and 5.0e-3 (bf16) on this graph and
# 1.5e-3 / 1.2e-2 on the five-scale MDX-Net graph below: 4-6x inside these bounds.
TOL = {"f32": 1e-5, "f16": 3e-3, "bf16": 3e-2}


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def run(torch, graph, x):
    return graph.forward(torch.from_numpy(np.asarray(x, np.float32)).cuda()).cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("mode", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("batch", [1, 2])
def test_graph_with_gemm_matches_oracle(torch_cuda, mode, batch):
    from ancha_b200.mdx import Graph
    from test_gpu_mdx import tfc_tdf_graph  # 3×3, 1×1, 2×2 / 2, grouped dilated conv, TDF MatMuls
    onnx, _ = tfc_tdf_graph()
    x = np.random.default_rng(3).standard_normal((batch, 4, 64, 32))
    ref = M.Graph(onnx, True).forward(x)
    y = run(torch_cuda, Graph(onnx, 0, True, gemm=mode), x)
    err = np.abs(y - ref).max() / np.abs(ref).max()
    print(f"classic MDX conv_gemm {mode} batch {batch}: max |d| / max |ref| {err:.2e}")
    assert y.shape == ref.shape and err < TOL[mode]


def test_gemm_off_restores_direct_kernels(torch_cuda):
    from ancha_b200.mdx import Graph
    from test_gpu_mdx import tfc_tdf_graph
    onnx, _ = tfc_tdf_graph()
    x = np.random.default_rng(4).standard_normal((1, 4, 64, 32))
    direct = run(torch_cuda, Graph(onnx, gemm=None), x)
    g = Graph(onnx, 0, True, gemm="f16")
    assert not np.array_equal(run(torch_cuda, g, x), direct)  # the 16-bit path did run
    N.check(N.lib().ancha_mdx_set_gemm(g._h, -1))
    assert np.array_equal(run(torch_cuda, g, x), direct)


@pytest.mark.parametrize("mode", ["f32", "bf16"])
def test_separate_task_with_gemm_matches_oracle(torch_cuda, mode):
    from ancha_b200.mdx import Graph
    from test_gpu_mdx import shape_preserving_graph
    onnx = shape_preserving_graph()
    x = (np.random.default_rng(7).standard_normal((2, 4000)) * 0.1).astype(np.float32)
    ref_p, _ = M.separate(M.Graph(onnx, True), 512, 256, 16, 1.035, x.astype(np.float64), hop=128, batch=2)
    p, r, _ = Graph(onnx, 0, True, gemm=mode).separate_pcm(x, n_fft=512, hop=128, bins=256, frames=16,
                                                            compensate=1.035, batch=2)
    err = np.abs(p - ref_p).max() / np.abs(ref_p).max()
    print(f"classic MDX task conv_gemm {mode}: max |d| / max |ref| {err:.2e}")
    assert err < {"f32": 2e-5, "bf16": 3e-2}[mode]
    assert np.abs(p + r - x).max() < 1e-6


@pytest.mark.parametrize("mode", [None, "f32", "bf16"])
def test_mdx_net_graph_matches_oracle(torch_cuda, mode):
    """The classic MDX-Net benchmark's network family at full depth (five scales) on a small tile."""
    from ancha_b200 import mdx_net as MN
    from ancha_b200.mdx import Graph
    c = MN.MdxNetConfig(dim_f=256, dim_t=64, growth=8, scales=5, layers=3, bottleneck=8)
    onnx = MN.tfc_tdf_v1(c, seed=0)
    x = np.random.default_rng(5).standard_normal((2, 4, c.dim_f, c.dim_t))
    ref = M.Graph(onnx, True).forward(x)
    y = run(torch_cuda, Graph(onnx, 0, True, gemm=mode), x)
    err = np.abs(y - ref).max() / np.abs(ref).max()
    print(f"TFC-TDF v1 conv_gemm {mode}: max |d| / max |ref| {err:.2e}")
    assert err < {None: 1e-5, "f32": 1e-5, "bf16": 5e-2}[mode]
