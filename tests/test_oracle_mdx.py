"""Classic MDX ONNX executor oracle against the reference's graph known answers
(crates/ancha-models/tests/mdx_contracts.rs), on graphs written by ancha_b200.onnx_writer."""
import numpy as np
import pytest

from ancha_b200.onnx_writer import Attr, Node, model
from oracle import mdx as M


def fold_graph():
    # mdx_contracts.rs:35-58: ConvTranspose(1 → 2, 1×1, bias) → BatchNormalization → Relu.
    return model([Node("ConvTranspose", ["x", "w", "bias"], "conv"),
                  Node("BatchNormalization", ["conv", "gamma", "beta", "mean", "var"], "bn"),
                  Node("Relu", ["bn"], "out")],
                 {"w": np.array([2.0, -1.0]).reshape(1, 2, 1, 1), "bias": np.array([0.25, -0.75]),
                  "gamma": np.array([1.5, 0.5]), "beta": np.array([0.4, -0.3]),
                  "mean": np.array([0.8, -1.2]), "var": np.array([0.5, 2.0])})


def test_transpose_bn_folding_matches_eval_reference():
    x = np.array([1.0, -2.0, 0.0, 4.0]).reshape(1, 1, 2, 2)
    reference, optimized = M.Graph(fold_graph(), False), M.Graph(fold_graph(), True)
    assert (reference.folded_bn, optimized.folded_bn) == (0, 1)
    a, b = reference.forward(x), optimized.forward(x)
    for c in range(2):
        for i, v in enumerate([1.0, -2.0, 0.0, 4.0]):
            e = max(((v * [2.0, -1.0][c] + [0.25, -0.75][c]) - [0.8, -1.2][c])
                    / np.sqrt(np.float32([0.5, 2.0][c]) + np.float32(1e-5)) * [1.5, 0.5][c] + [0.4, -0.3][c], 0.0)
            assert abs(a.ravel()[c * 4 + i] - e) < 2e-6
            assert abs(b.ravel()[c * 4 + i] - e) < 2e-6


def chain_graph():
    # mdx_contracts.rs:90-113: MatMul → Add (skip) → Transpose(0, 1, 3, 2) → Mul → 1×1 Conv.
    return model([Node("MatMul", ["x", "matrix"], "product"), Node("Add", ["product", "x"], "sum"),
                  Node("Transpose", ["sum"], "transposed", attrs=[Attr("perm", ints=[0, 1, 3, 2])]),
                  Node("Mul", ["transposed", "scale"], "scaled"), Node("Conv", ["scaled", "w"], "out")],
                 {"matrix": np.array([[1.0, 2.0], [3.0, 4.0]]), "scale": np.array([0.5]),
                  "w": np.array([2.0]).reshape(1, 1, 1, 1)})


def test_nchw_matmul_broadcast_transpose_conv_and_skip_values():
    g = M.Graph(chain_graph(), True)
    assert g.forward(np.array([1.0, 2.0, 3.0, 4.0]).reshape(1, 1, 2, 2)).ravel().tolist() == [8, 18, 12, 26]
    batched = np.arange(1.0, 9.0).reshape(2, 1, 2, 2)
    assert g.forward(batched).ravel().tolist() == [8, 18, 12, 26, 28, 38, 40, 54]


def test_graph_rejects_unknown_ops_nonfinite_constants_and_cancels():
    # mdx_contracts.rs:133-166.
    ok = model([Node("Relu", ["x"], "out")], {})
    g = M.Graph(ok, True)
    with pytest.raises(M.GraphError):
        g.forward(np.zeros((1, 1, 1, 1)), cancelled=True)
    with pytest.raises(M.GraphError):
        M.Graph(model([Node("Sigmoid", ["x"], "out")], {}), True)
    with pytest.raises(M.GraphError):
        M.Graph(model([Node("Relu", ["x"], "out")], {"invalid": np.array([np.nan])}), True)


def test_structural_rejections():
    relu = [Node("Relu", ["x"], "out")]
    with pytest.raises(M.GraphError):
        M.Graph(model(relu, {}, opset=12), True)  # opset 13 only
    with pytest.raises(M.GraphError):
        M.Graph(model(relu, {}, outputs=("out", "other")), True)  # one output
    with pytest.raises(M.GraphError):
        M.Graph(model([Node("Conv", ["x", "w"], "out", attrs=[Attr("pads", ints=[1, 0, 0, 0])])],
                      {"w": np.ones((1, 1, 3, 3))}), True)  # asymmetric pads
    with pytest.raises(M.GraphError):
        M.Graph(model([Node("Relu", ["y"], "out")], {}), True)  # unknown input
    with pytest.raises(M.GraphError):
        M.Graph(model([Node("Conv", ["x", "w"], "out", attrs=[Attr("auto_pad", i=1)])],
                      {"w": np.ones((1, 1, 1, 1))}), True)  # attribute outside the allow-list


def test_grouped_dilated_strided_convolutions_match_direct_sums():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 4, 7, 9))
    w = rng.standard_normal((6, 2, 3, 2))
    y = M.conv2d(x, w, (2, 1), (1, 2), (2, 1), 2)
    oh, ow = y.shape[2:]
    xp = np.pad(x, ((0, 0), (0, 0), (1, 1), (2, 2)))
    for b in range(2):
        for o in range(6):
            g = o // 3
            for i in range(oh):
                for j in range(ow):
                    acc = 0.0
                    for c in range(2):
                        for ky in range(3):
                            for kx in range(2):
                                acc += xp[b, g * 2 + c, i * 2 + ky * 2, j + kx] * w[o, c, ky, kx]
                    assert abs(y[b, o, i, j] - acc) < 1e-10
    wt = rng.standard_normal((4, 3, 2, 3))
    z = M.conv_transpose2d(x, wt, (2, 2), (1, 0), (1, 0), (1, 2), 2)
    full = np.zeros((2, 6, 6 * 2 + 2 + 1, 8 * 2 + 4 + 1))
    for b in range(2):
        for ci in range(4):
            g = ci // 2
            for i in range(7):
                for j in range(9):
                    for o in range(3):
                        for ky in range(2):
                            for kx in range(3):
                                full[b, g * 3 + o, i * 2 + ky, j * 2 + kx * 2] += x[b, ci, i, j] * wt[ci, o, ky, kx]
    assert np.abs(z - full[:, :, 1:1 + z.shape[2], 0:z.shape[3]]).max() < 1e-10


# ---- The library's C++ reader / graph builder (host-only ABI) against the oracle ----------

def _lib_inspect(b, optimized=True):
    from ancha_b200 import mdx
    return mdx.inspect(b, optimized)


@pytest.mark.parametrize("optimized", [False, True])
def test_library_graph_builder_matches_oracle(optimized):
    for g in (fold_graph(), chain_graph()):
        o = M.Graph(g, optimized)
        info = _lib_inspect(g, optimized)
        assert info == {"nodes": o.nodes, "instructions": len(o.instructions), "folded_bn": o.folded_bn,
                        "constants": len(o.constants)}
    assert _lib_inspect(fold_graph(), optimized)["folded_bn"] == (1 if optimized else 0)


def _tensor_bytes(name, dims, floats=0):
    """A FLOAT TensorProto with arbitrary dims and `floats` zero values of raw data."""
    from ancha_b200 import onnx_writer as W
    out = b"".join(W._int(1, d) for d in dims) + W._int(2, W.FLOAT) + W._str(8, name)
    return out + W._len(9, bytes(4 * min(floats, 16)))


def test_library_graph_builder_rejections():
    from ancha_b200 import _native as N
    cases = [
        (model([Node("Sigmoid", ["x"], "out")], {}), "unsupported ONNX operation"),
        (model([Node("Relu", ["x"], "out")], {"invalid": np.array([np.nan])}), "invalid initializer"),
        (model([Node("Relu", ["x"], "out")], {}, opset=12), "opset 13"),
        (model([Node("Relu", ["x"], "out")], {}, outputs=("out", "other")), "one input and one output"),
        (model([Node("Conv", ["x", "w"], "out", attrs=[Attr("pads", ints=[1, 0, 0, 0])])],
               {"w": np.ones((1, 1, 3, 3))}), "asymmetric"),
        (model([Node("Relu", ["y"], "out")], {}), "unknown input"),
        (model([Node("Conv", ["x", "w"], "out", attrs=[Attr("auto_pad", i=1)])], {"w": np.ones((1, 1, 1, 1))}),
         "unsupported attribute"),
        (model([Node("Transpose", ["x"], "out", attrs=[Attr("perm", ints=[0, 1, 1, 2])])], {}), "permutation"),
        (b"\x0a\xff", "truncated"),
        # dims whose product wraps a 64-bit count to 0 = the length of its empty data
        (model([Node("Relu", ["x"], "out")], {}, raw_tensors=[_tensor_bytes("wrap", [1 << 32, 1 << 32])]),
         "invalid initializer"),
        (model([Node("Relu", ["x"], "out")], {}, raw_tensors=[_tensor_bytes("big", [1 << 31], 1 << 31)]),
         "invalid initializer"),  # one dim past 2^30, with no data behind it
    ]
    for g, msg in cases:
        with pytest.raises(N.AnchaError) as e:
            _lib_inspect(g)
        assert e.value.status == N.E_INVALID and msg in str(e.value), (msg, str(e.value))
        if g != b"\x0a\xff":
            with pytest.raises(M.GraphError):
                M.Graph(g, True)


def test_mdx_packing_zeroes_low_bins_and_pads_frequency():
    # mdx_dsp_contracts.rs:6-41: for n_fft 5120 and 6144, pack then unpack equals the inverse
    # STFT of the spectrum with bins < 3 and bins >= 2048 zeroed.
    from oracle.dsp import Stft
    n = 10240
    planes = np.stack([np.sin(np.arange(n) * (0.015 + c * 0.09)) * 0.1 for c in range(2)])
    for fft in (5120, 6144):
        st = Stft(fft, 1024)
        packed = M.pack(st, planes, 2048)
        assert packed.shape == (4, 2048, n // 1024 + 1)
        actual = M.unpack(st, packed, n)
        for c in range(2):
            z = st.forward(planes[c]).copy()
            z[:, :3] = 0
            z[:, 2048:] = 0
            assert np.abs(actual[c] - st.inverse(z, n, False)).max() < 1e-7


def test_mdx_separate_identity_graph_reconstructs_and_rejects_bad_options():
    # An identity graph (a 1×1 Conv with the identity as weight) turns separate into STFT →
    # iSTFT → weighted overlap-add: tones well above the three zeroed bins come back up to the
    # chunk-edge effects of those bins, and predicted + residual is the input exactly.
    g = M.Graph(model([Node("Conv", ["x", "w"], "out")], {"w": np.eye(4).reshape(4, 4, 1, 1)}), True)
    n = 5000
    x = np.stack([np.sin(np.arange(n) * 0.3), np.cos(np.arange(n) * 0.21)]) * 0.2
    for overlap in (None, 0.0, 0.5):
        pred, res = M.separate(g, n_fft=512, bins=256, frames=16, compensate=1.0, planes=x, hop=128,
                               overlap=overlap)
        assert np.abs(pred + res - x).max() < 1e-12
        assert np.abs(pred - x).max() < 0.03
        if overlap != 0.0:  # Hann-weighted chunks blend the edges away from the track ends
            assert np.abs(pred - x)[:, 200:-200].max() < 1e-3
    pred2, _ = M.separate(g, 512, 256, 16, 1.035, x, hop=128, denoise=True)
    pred1, _ = M.separate(g, 512, 256, 16, 1.0, x, hop=128)
    assert np.abs(pred2 - 1.035 * pred1).max() < 1e-10  # the identity graph is odd: denoise keeps it
    for bad in (dict(overlap=0.99), dict(batch=0), dict(batch=5)):
        with pytest.raises(M.GraphError):
            M.separate(g, 512, 256, 16, 1.0, x, hop=128, **bad)


def test_graph_rejects_unknown_gemm_precision_before_loading():
    from ancha_b200 import _native as N
    from ancha_b200.mdx import Graph
    with pytest.raises(N.AnchaError) as e:
        Graph(chain_graph(), 0, True, gemm="f8")
    assert e.value.status == N.E_INVALID


def test_reader_accepts_both_protobuf_encodings():
    """onnx.proto is proto2: INTS attributes arrive unpacked from most writers, packed from some,
    and initializers as raw_data or packed float_data. Every combination builds the same graph
    and, in the oracle, computes the same values."""
    x = np.random.default_rng(1).standard_normal((1, 2, 5, 4))
    w = {"w": np.random.default_rng(2).standard_normal((3, 2, 3, 3)), "b": np.array([0.1, -0.2, 0.3])}
    outs = []
    for packed in (True, False):
        for float_data in (False, True):
            g = model([Node("Conv", ["x", "w", "b"], "c", attrs=[Attr("pads", ints=[1, 1, 1, 1], packed=packed),
                                                               Attr("strides", ints=[1, 2], packed=packed)]),
                       Node("Transpose", ["c"], "out", attrs=[Attr("perm", ints=[0, 1, 3, 2], packed=packed)])],
                      w, float_data=float_data)
            assert _lib_inspect(g) == {"nodes": 2, "instructions": 2, "folded_bn": 0, "constants": 2}
            outs.append(M.Graph(g).forward(x))
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])
    assert outs[0].shape == (1, 3, 2, 5)
