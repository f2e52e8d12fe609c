"""MDX23C oracle pinned to the reference's golden PyTorch forward and known-answer tests
(crates/ancha-models/tests/mdx23c_contracts.rs, tests/mdx23c_runtime_contracts.rs)."""
import json
import os

import numpy as np
import pytest

from oracle import mdx23c as M

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "mdx23c_tiny.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


def test_weight_inventory_matches_fixture(golden):
    shapes = M.weight_shapes(golden["config"])
    assert len(shapes) == 80  # tensor_count of mdx23c_contracts.rs:20
    assert shapes == {w["name"]: tuple(w["shape"]) for w in golden["weights"]}


def test_forward_matches_pytorch_golden(golden):
    c = golden["config"]
    M.validate(c)
    w = M.fixture_weights([(x["name"], x["shape"]) for x in golden["weights"]])
    y = M.forward(c, w, M.fixture_input(golden["input_shape"]))
    e = np.array(golden["expected"]).reshape(golden["output_shape"])
    assert y.shape == tuple(golden["output_shape"])
    # The reference gates at relative MSE 1e-8 and max |Δ| 1e-5 (mdx23c_contracts.rs:42-49).
    assert ((y - e) ** 2).sum() / (e ** 2).sum() < 1e-12
    assert np.abs(y - e).max() < 1e-9


def test_forward_rejects_bad_shapes(golden):
    c = golden["config"]
    w = M.fixture_weights([(x["name"], x["shape"]) for x in golden["weights"]])
    with pytest.raises(ValueError):
        M.forward(c, w, np.zeros((1, 4, 32, 7), np.float32))  # frames not a multiple of 4
    with pytest.raises(ValueError):
        M.forward(c, w, np.zeros((5, 4, 32, 8), np.float32))  # batch above 4
    with pytest.raises(ValueError):
        M.forward(c, w, np.zeros((1, 2, 32, 8), np.float32))


def test_transpose_convolution_keeps_batch_channel_and_spatial_phases():
    # mdx23c_contracts.rs:77-135, including the non-square 2 × 3 kernel.
    for b, ci, co, h, wd, kh, kw in [(2, 3, 2, 3, 5, 2, 2), (1, 2, 3, 2, 4, 2, 3)]:
        x = np.sin(np.arange(b * ci * h * wd) * 0.13).reshape(b, ci, h, wd)
        wt = (np.cos(np.arange(ci * co * kh * kw) * 0.07) * 0.1).reshape(ci, co, kh, kw)
        y = M.conv_transpose2x2(x, wt)
        e = np.zeros((b, co, h * kh, wd * kw))
        for bb in range(b):
            for o in range(co):
                for yy in range(h):
                    for z in range(wd):
                        for ky in range(kh):
                            for kx in range(kw):
                                e[bb, o, yy * kh + ky, z * kw + kx] = sum(
                                    x[bb, i, yy, z] * wt[i, o, ky, kx] for i in range(ci))
        assert np.abs(y - e).max() < 1e-12


def test_instance_norm_epsilon_and_biased_variance():
    # mdx23c_contracts.rs:137-155.
    v = 1e-4 * np.sin(np.arange(24.0)).reshape(2, 2, 2, 3)
    g, b = np.array([1.2, -0.7]), np.array([0.01, -0.03])
    y = M.instance_norm(v, g, b)
    for n in range(2):
        for c in range(2):
            x = v[n, c].ravel()
            mean = x.mean()
            var = ((x - mean) ** 2).mean()
            assert np.allclose(y[n, c].ravel(), (x - mean) / np.sqrt(var + 1e-5) * g[c] + b[c], atol=1e-12)


def test_config_rejects_shapes_that_cannot_survive_all_scales():
    # mdx23c_contracts.rs:157-176.
    native = M.inst_voc_hq2()
    M.validate(native)
    assert M.chunk_samples(native) == 261120
    for change in range(7):
        c = dict(native)
        if change == 0: c["frames"] = 255
        elif change == 1: c["bins"] = 4095
        elif change == 2: c["subbands"] = 0
        elif change == 3: c["overlap"] = 0
        elif change == 4: c["scales"] = 0
        elif change == 5: c["stems"] = ["instrumental", "vocals"]
        else: c["bottleneck_factor"] = 0
        with pytest.raises(ValueError):
            M.validate(c)


def test_uvr_overlap_plan_reconstructs_boundaries():
    # mdx23c_runtime_contracts.rs:16-47.
    p = M.OverlapPlan(132300, 261120, 8)
    assert (p.step, p.border, p.pad, p.chunks) == (32640, 228480, 30900, 12)
    with pytest.raises(ValueError):
        M.OverlapPlan(0, 128, 8)
    for n in [1, 32, 127, 128, 129, 256, 333]:
        for overlap in [1, 2, 4, 8]:
            p = M.OverlapPlan(n, 128, overlap)
            x = (np.arange(n) * 0.001 + 0.1).astype(np.float32)[None]
            y = np.zeros(n)
            for i in range(p.chunks):
                s = i * p.step
                wave = p.window(x, s)
                lo, hi = max(s, p.border), min(s + p.chunk, p.border + n)
                y[lo - p.border:hi - p.border] += wave[0, lo - s:hi - s]
            assert np.abs(y / overlap - x[0]).max() < 1e-6


def test_spectral_packing_retains_dc_and_stereo_complex_order():
    # mdx23c_runtime_contracts.rs:49-64: constant planes 0.25 / -0.125, n_fft 64, hop 8.
    from oracle.dsp import Stft
    st = Stft(64, 8)
    planes = np.stack([np.full(56, 0.25), np.full(56, -0.125)])
    p = M.pack(st, planes, 32)
    assert p.shape == (4, 32, 8)
    assert abs(p.ravel()[0] - 8.0) < 1e-6
    assert abs(p.ravel()[2 * 32 * 8] + 4.0) < 1e-6
    assert np.abs(M.unpack(st, p, 56) - planes).max() < 1e-6


def test_separate_length_and_chunk_skipping(golden):
    c = golden["config"]
    w = M.fixture_weights([(x["name"], x["shape"]) for x in golden["weights"]])
    x = np.random.default_rng(0).standard_normal((2, 300)) * 0.1
    y = M.separate(c, w, x)
    assert y.shape == (2, 2, 300) and np.isfinite(y).all()
    # Chunks entirely inside the zero borders contribute nothing: skipping them is exact.
    assert np.array_equal(y, M.separate(c, w, x, optimized=False))
