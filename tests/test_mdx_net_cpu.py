"""The synthetic classic MDX-Net graph (ancha_b200/mdx_net.py, the classic MDX-Net benchmark workload) on
the CPU: the library's graph builder and the oracle agree on its structure, the oracle runs it
with bounded activations, BatchNormalization folding does not change it, and forward_flops
equals the multiply-adds the oracle performs."""
import numpy as np
import pytest

from ancha_b200 import mdx, mdx_net as MN
from oracle import mdx as M

TINY = MN.MdxNetConfig(dim_f=64, dim_t=32, growth=4, scales=3, layers=2, bottleneck=4)


def test_structure_matches_oracle():
    g = MN.tfc_tdf_v1(TINY, seed=1)
    for optimized in (False, True):
        o = M.Graph(g, optimized)
        assert mdx.inspect(g, optimized) == {"nodes": o.nodes, "instructions": len(o.instructions),
                                             "folded_bn": o.folded_bn, "constants": len(o.constants)}
    # one ConvTranspose + BatchNormalization pair per decoder level folds
    assert mdx.inspect(g, True)["folded_bn"] == TINY.scales


def test_forward_is_bounded_and_folding_is_exact():
    g = MN.tfc_tdf_v1(TINY, seed=2)
    x = np.random.default_rng(0).standard_normal((2, 4, TINY.dim_f, TINY.dim_t))
    y = M.Graph(g, True).forward(x)
    assert y.shape == x.shape and np.isfinite(y).all()
    assert 1e-3 < np.sqrt((y ** 2).mean()) < 1e2
    assert np.abs(y - M.Graph(g, False).forward(x)).max() <= 1e-9 * np.abs(y).max()


def test_forward_flops_counts_the_oracle_multiply_adds(monkeypatch):
    macs = [0]
    conv, convt, matmul = M.conv2d, M.conv_transpose2d, np.matmul

    def counted_conv(x, w, *a, **k):
        y = conv(x, w, *a, **k)
        macs[0] += y.size * w.shape[1] * w.shape[2] * w.shape[3]
        return y

    def counted_convt(x, w, *a, **k):
        macs[0] += x.size * w.shape[1] * w.shape[2] * w.shape[3]  # every input meets co·kh·kw taps
        return convt(x, w, *a, **k)

    def counted_matmul(a, b):
        y = matmul(a, b)
        macs[0] += y.size * a.shape[-1]
        return y

    monkeypatch.setattr(M, "conv2d", counted_conv)
    monkeypatch.setattr(M, "conv_transpose2d", counted_convt)
    monkeypatch.setattr(M.np, "matmul", counted_matmul)
    g = MN.tfc_tdf_v1(TINY, seed=3)
    M.Graph(g, True).forward(np.zeros((1, 4, TINY.dim_f, TINY.dim_t)))
    assert 2 * macs[0] == MN.forward_flops(TINY)


def test_config_rejects_shapes_that_do_not_survive_the_scales():
    with pytest.raises(ValueError):
        MN.tfc_tdf_v1(MN.MdxNetConfig(dim_f=96, dim_t=32, scales=5))
