"""MDX23C on the GPU through the C ABI against the reference's golden PyTorch forward and
the numpy oracle (oracle/mdx23c.py): f32 to the golden's precision, f16 / bf16 by SNR, plus
shape, cancellation and checksum errors."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from ancha_b200 import _native as N
from ancha_b200.mdx23c import Mdx23c, write_package
from oracle import mdx23c as M

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "mdx23c_tiny.json")
# SNR floors (dB) for the reduced-precision paths: f16 / bf16 GEMM operands, f32 accumulation
# and f32 activations between layers.
SNR_FLOOR = {"f16": 45.0, "bf16": 30.0}


def snr_db(ref, out):
    ref = np.asarray(ref, np.float64)
    err = np.asarray(out, np.float64) - ref
    return 10 * np.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


@pytest.fixture(scope="module")
def golden(tmp_path_factory):
    with open(GOLDEN) as f:
        g = json.load(f)
    w = M.fixture_weights([(x["name"], x["shape"]) for x in g["weights"]])
    d = str(tmp_path_factory.mktemp("mdx23c_tiny"))
    write_package(d, g["config"], w)
    return g, w, d


def mid_config():
    """Three scales, two blocks per scale, channel counts that meet the tensor-core GEMM's
    16-byte rules, and a bottleneck TDF (K = 4) that does not."""
    return dict(family="mdx23c", sample_rate=44100, n_fft=512, hop=128, bins=256, frames=32, overlap=4,
                subbands=2, channels=32, growth=16, scales=3, blocks_per_scale=2, bottleneck_factor=4,
                scale=[2, 2], stems=["vocals", "instrumental"])


@pytest.fixture(scope="module")
def mid(tmp_path_factory):
    c = mid_config()
    M.validate(c)
    rng = np.random.default_rng(7)
    w = {}
    for name, shape in sorted(M.weight_shapes(c).items()):
        if len(shape) == 1 and name.endswith("weight"):
            w[name] = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        elif len(shape) == 1:
            w[name] = (0.1 * rng.standard_normal(shape)).astype(np.float32)
        else:
            fan_in = int(np.prod(shape[1:]))
            w[name] = (rng.standard_normal(shape) / np.sqrt(fan_in)).astype(np.float32)
    d = str(tmp_path_factory.mktemp("mdx23c_mid"))
    write_package(d, c, w)
    return c, w, d


def test_golden_forward_f32(torch_cuda, golden):
    g, _, d = golden
    m = Mdx23c(d, 0, "f32")
    assert m.tensor_count == 80
    x = torch_cuda.from_numpy(M.fixture_input(g["input_shape"])).cuda()
    y = m.forward(x).cpu().numpy().astype(np.float64)
    e = np.array(g["expected"]).reshape(g["output_shape"])
    assert y.shape == e.shape
    rel_mse = ((y - e) ** 2).sum() / (e ** 2).sum()
    print(f"golden f32: rel MSE {rel_mse:.3e}, max |d| {np.abs(y - e).max():.3e}")
    # The reference gates its own f32 forward at rel MSE 1e-8, max |d| 1e-5.
    assert rel_mse < 1e-10
    assert np.abs(y - e).max() < 1e-9


@pytest.mark.parametrize("precision", ["f16", "bf16"])
def test_golden_forward_reduced_precision(torch_cuda, golden, precision):
    g, w, d = golden
    x = M.fixture_input(g["input_shape"])
    ref = M.forward(g["config"], w, x)
    y = Mdx23c(d, 0, precision).forward(torch_cuda.from_numpy(x).cuda()).cpu().numpy()
    s = snr_db(ref, y)
    print(f"golden {precision}: {s:.1f} dB")
    assert s >= SNR_FLOOR[precision]


@pytest.mark.parametrize("precision", ["f32", "f16", "bf16"])
def test_mid_network_matches_oracle(torch_cuda, mid, precision):
    c, w, d = mid
    rng = np.random.default_rng(11)
    x = rng.standard_normal((1, 4, c["bins"], c["frames"])).astype(np.float32)
    ref = M.forward(c, w, x)
    y = Mdx23c(d, 0, precision).forward(torch_cuda.from_numpy(x).cuda()).cpu().numpy()
    s = snr_db(ref, y)
    err = np.abs(y - ref).max() / np.abs(ref).max()
    print(f"mid {precision}: {s:.1f} dB, max |d| / max |ref| {err:.2e}")
    if precision == "f32":
        assert err < 1e-5
    else:
        assert s >= SNR_FLOOR[precision]


def wide_config():
    """Planes 1024 / 512 / 256 wide with channels in 64s: every 3 × 3 and 1 × 1 layer of the
    16-bit paths runs as an implicit GEMM, with 256-position tiles inside one row."""
    return dict(family="mdx23c", sample_rate=44100, n_fft=2048, hop=256, bins=1024, frames=8, overlap=4,
                subbands=1, channels=64, growth=64, scales=2, blocks_per_scale=1, bottleneck_factor=4,
                scale=[2, 2], stems=["vocals", "instrumental"])


@pytest.mark.parametrize("precision", ["f32", "f16", "bf16"])
def test_wide_network_matches_oracle(torch_cuda, tmp_path, precision):
    from ancha_b200.mdx23c import random_tensors
    c = wide_config()
    M.validate(c)
    w = random_tensors(c, seed=3)
    write_package(str(tmp_path), c, w)
    x = np.random.default_rng(13).standard_normal((1, 4, c["bins"], c["frames"])).astype(np.float32)
    ref = M.forward(c, w, x)
    y = Mdx23c(str(tmp_path), 0, precision).forward(torch_cuda.from_numpy(x).cuda()).cpu().numpy()
    s = snr_db(ref, y)
    print(f"wide {precision}: {s:.1f} dB")
    if precision == "f32":
        assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-5
    else:
        assert s >= SNR_FLOOR[precision]


@pytest.mark.parametrize("precision", ["f16", "bf16"])
def test_full_size_reduced_precision_against_f32(torch_cuda, tmp_path, precision):
    """inst_voc_hq2 at its native size (the benchmarked network, synthetic weights): the
    16-bit implicit-GEMM forward against this library's f32 forward (FFMA GEMMs and patch
    matrices, checked against the oracle above), a size-independent SNR check."""
    from ancha_b200.mdx23c import inst_voc_hq2, random_tensors
    c = inst_voc_hq2()
    write_package(str(tmp_path), c, random_tensors(c, seed=1))
    x = torch_cuda.randn(1, 4, c["bins"], c["frames"], generator=torch_cuda.Generator().manual_seed(2)).cuda()
    ref = Mdx23c(str(tmp_path), 0, "f32").forward(x).cpu().numpy()
    y = Mdx23c(str(tmp_path), 0, precision).forward(x).cpu().numpy()
    assert np.isfinite(y).all()
    s = snr_db(ref, y)
    print(f"inst_voc_hq2 {precision} vs f32: {s:.1f} dB")
    assert s >= SNR_FLOOR[precision]


def test_batch_and_frame_count_other_than_the_manifest(torch_cuda, mid):
    c, w, d = mid
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 4, c["bins"], 16)).astype(np.float32)  # batch 2, 16 of 32 frames
    ref = M.forward(c, w, x)
    y = Mdx23c(d, 0, "f32").forward(torch_cuda.from_numpy(x).cuda()).cpu().numpy()
    assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-5


def test_shape_errors_and_cancellation(torch_cuda, golden):
    g, _, d = golden
    m = Mdx23c(d, 0, "f32")
    for shape in [(1, 4, 32, 7), (5, 4, 32, 8)]:  # frames not a multiple of 4; batch above 4
        with pytest.raises(N.AnchaError) as e:
            m.forward(torch_cuda.zeros(shape, device="cuda"))
        assert e.value.status == N.E_INVALID
    with pytest.raises(N.AnchaError) as e:
        m.forward(torch_cuda.zeros((1, 4, 32, 8), device="cuda"), cancel=C.c_int(1))
    assert e.value.status == N.E_CANCELLED


def test_corrupt_checksum_is_rejected(torch_cuda, golden, tmp_path):
    g, w, _ = golden
    d = str(tmp_path / "corrupt")
    man = write_package(d, g["config"], w)
    man["weights_sha256"] = "0" * 64
    with open(os.path.join(d, "manifest.json"), "w") as fh:
        json.dump(man, fh)
    with pytest.raises(N.AnchaError) as e:
        Mdx23c(d, 0, "f32")
    assert "checksum" in str(e.value)


def test_separate_pcm_tiny_matches_oracle(torch_cuda, golden):
    """The whole task on the device (UVR chunks, STFT 64 / hop 8, network, iSTFT, overlap-add)
    against the oracle's restatement of mdx23c_runtime::separate."""
    g, w, d = golden
    x = (np.random.default_rng(1).standard_normal((2, 300)) * 0.1).astype(np.float32)
    ref = M.separate(g["config"], w, x)
    for batch in (1, 3):
        y, secs = Mdx23c(d, 0, "f32").separate_pcm(x, batch=batch)
        assert y.shape == ref.shape and secs > 0
        err = np.abs(y - ref).max() / np.abs(ref).max()
        print(f"separate tiny batch {batch}: max |d| / max |ref| {err:.2e}")
        assert err < 1e-5


@pytest.mark.parametrize("precision", ["f32", "f16"])
def test_separate_pcm_mid_matches_oracle(torch_cuda, mid, precision):
    c, w, d = mid  # n_fft 512, hop 128, 3968-sample chunks, overlap 4
    x = (np.random.default_rng(2).standard_normal((2, 6000)) * 0.1).astype(np.float32)
    ref = M.separate(c, w, x)
    y, _ = Mdx23c(d, 0, precision).separate_pcm(x)
    s = snr_db(ref, y)
    print(f"separate mid {precision}: {s:.1f} dB")
    if precision == "f32":
        assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-5
    else:
        assert s >= SNR_FLOOR[precision]


def test_separate_pcm_cancel_and_shape_errors(torch_cuda, golden):
    _, _, d = golden
    m = Mdx23c(d, 0, "f32")
    x = np.zeros((2, 300), np.float32)
    with pytest.raises(N.AnchaError) as e:
        m.separate_pcm(x, cancel=C.c_int(1))
    assert e.value.status == N.E_CANCELLED
    with pytest.raises(N.AnchaError):
        m.separate_pcm(np.zeros((1, 300), np.float32))
