"""The oracle pinned against the reference's own known answers and invariants.

Each test replays a contract of the reference's test suite on the numpy oracle:
``crates/ancha-audio/tests/audio_contracts.rs``, ``crates/ancha-kernels/tests/contracts.rs``
and ``crates/ancha-models/tests/model_contracts.rs``.
"""
import math

import numpy as np
import pytest

from oracle import dsp, kernels, roformer


def signal(n):
    i = np.arange(n, dtype=np.float32)
    return ((np.sin(i * np.float32(0.071)) + np.float32(0.2) * np.cos(i * np.float32(0.31)))
            * np.float32(0.4)).astype(np.float32)


@pytest.mark.parametrize("hop", [441, 512])
@pytest.mark.parametrize("n", [1025, 2048, 4103, 88201])
def test_stft_round_trip_edges_odd_lengths(hop, n):
    # audio_contracts.rs:16-35
    stft = dsp.Stft(2048, hop)
    x = signal(n)
    x[0], x[n - 1] = 0.81, -0.72
    spec = stft.forward(x)
    assert spec.shape[0] == n // hop + 1
    y = stft.inverse(spec, n, False)
    assert y.shape[0] == n
    assert np.max(np.abs(x - y)) < 2e-6


def test_stft_matches_analytical_centered_periodic_hann_dc():
    # audio_contracts.rs:38-49
    stft = dsp.Stft(2048, 512)
    spec = stft.forward(np.ones(4096, dtype=np.float32))
    assert abs(spec[0, 0].real - 1024.0) < 1e-3
    assert abs(spec[0, 1].real + 512.0) < 1e-3
    assert abs(spec[0, 2]) < 1e-3
    assert np.all(np.isfinite(stft.inverse(spec, 4096, True)))
    with pytest.raises(ValueError):
        dsp.Stft(2047, 512)
    with pytest.raises(ValueError):
        stft.forward(np.zeros(1024, dtype=np.float32))
    with pytest.raises(ValueError):
        stft.forward(np.full(2048, np.nan, dtype=np.float32))


def test_reflect_padding_excludes_edge_and_repeats():
    # audio_contracts.rs:52-56
    assert [dsp.reflect_index(i, 4) for i in range(-4, 8)] == [2, 3, 2, 1, 0, 1, 2, 3, 2, 1, 0, 1]
    assert dsp.reflect_index(-5, 1) == 0
    assert list(dsp.reflect_indices(np.arange(-4, 8), 4)) == [2, 3, 2, 1, 0, 1, 2, 3, 2, 1, 0, 1]


@pytest.mark.parametrize("n", [1, 31, 64, 65, 128, 303])
@pytest.mark.parametrize("overlap", [1, 2, 4])
def test_overlap_add_identity_at_every_boundary(n, overlap):
    # audio_contracts.rs:59-89
    plan = dsp.ChunkPlan(64, overlap)
    x = signal(n)
    acc = dsp.Accumulator(2, n)
    for start in plan.starts(n):
        c = np.array([x[start + i] if start + i < n else 0.0 for i in range(64)])
        acc.add(plan, start, np.stack([c, -c]))
    out = acc.finish()
    assert np.all(np.abs(x - out[0]) < 1e-6)
    assert np.all(np.abs(x + out[1]) < 1e-6)


def test_overlap_add_rejects_bad_plans():
    with pytest.raises(ValueError):
        dsp.ChunkPlan(64, 0)
    with pytest.raises(ValueError):
        dsp.Accumulator(2, 4).finish()


def test_chunk_weight_matches_scalar_rule():
    plan = dsp.ChunkPlan(100, 4)
    for first in (False, True):
        for last in (False, True):
            w = plan.weights(100, first, last)
            assert np.allclose(w, [plan.weight(i, first, last) for i in range(100)])


def values(n, shift):
    i = np.arange(n)
    return np.sin((i * 17 + shift).astype(np.float32) * np.float32(0.13))


@pytest.mark.parametrize("shape", [(1, 1, 1, 1), (19, 23, 7, 5), (33, 37, 64, 64)])
def test_online_softmax_matches_dense(shape):
    # contracts.rs:14-32
    nq, nk, d, dv = shape
    q, k, v = values(2 * nq * d, 1), values(2 * nk * d, 2), values(2 * nk * dv, 3)
    a = kernels.dense(q, k, v, 2, nq, nk, d, dv)
    for qt, kt in [(1, 1), (8, 7), (64, 128)]:
        b = kernels.tiled(q, k, v, 2, nq, nk, d, dv, qt, kt)
        assert np.all(np.abs(a - b) < 2e-5)


def test_attention_rejects_empty_nonfinite_and_zero_tiles():
    # contracts.rs:34-47
    with pytest.raises(ValueError):
        kernels.tiled([1.0], [1.0], [1.0], 1, 1, 1, 1, 1, 0, 1)
    with pytest.raises(ValueError):
        kernels.dense([np.nan], [1.0], [1.0], 1, 1, 1, 1, 1)
    with pytest.raises(ValueError):
        kernels.dense([], [1.0], [1.0], 1, 1, 1, 1, 1)


def test_norm_epsilon_semantics():
    # contracts.rs:49-55
    s, y = kernels.residual_l2norm([0, 0, 1e-14, 0], [0] * 4, [1, 1], 2, 2, 1e-12)
    assert list(s[:2]) == [0, 0] and list(y[:2]) == [0, 0]
    assert abs(y[2] - 0.01 * math.sqrt(2)) < 1e-6


def test_source_norm_known_answers():
    # model_contracts.rs:70-88: [3,4]·gamma[1,2]·sqrt(2); 1e-14 row → 0.01·sqrt(2); zeros stay 0.
    x = np.array([[0.0, 0.0], [1e-14, 0.0], [3.0, 4.0]])
    y = roformer.unit_norm(x) * (np.array([1.0, 2.0]) * math.sqrt(2))
    assert list(y[0]) == [0.0, 0.0]
    assert abs(y[1, 0] - 0.01 * math.sqrt(2)) < 1e-6
    assert abs(y[2, 0] - 0.6 * math.sqrt(2)) < 1e-6
    assert abs(y[2, 1] - 0.8 * 2 * math.sqrt(2)) < 1e-6


def test_pack_keeps_gate_bias_and_fold_is_columnwise():
    # contracts.rs:57-64
    w, b = kernels.pack_qkv_gate([1, 2, 3, 4, 5, 6], [7, 8], [0.5], 2)
    assert list(b) == [0, 0, 0, 0.5]
    f = kernels.fold_norm_scale(w, [2, 3])
    assert abs(f[6] - 7 * 2 * math.sqrt(2)) < 1e-5
    assert abs(f[7] - 8 * 3 * math.sqrt(2)) < 1e-5


def test_complex_multiplication_keeps_phase():
    # contracts.rs:66-71
    assert list(kernels.complex_mask_interleaved([1, 2, 3, -1], [4, 5, 0, 1])) == [-6, 13, 1, 3]


def test_rope_tables_match_reference_layout():
    # roformer.rs:155-175: cos pairs, sin pairs (-s, +s), query table scaled by 1/sqrt(d).
    freqs = np.array([1.0, 0.5], dtype=np.float32)
    cos, sin = roformer.rope_tables(freqs, 3, 0.5)
    assert cos.shape == (3, 4)
    assert np.allclose(cos[2], 0.5 * np.cos([2.0, 2.0, 1.0, 1.0]))
    assert np.allclose(sin[2], 0.5 * np.array([-np.sin(2.0), np.sin(2.0), -np.sin(1.0), np.sin(1.0)]))
    x = np.arange(8, dtype=np.float64).reshape(1, 2, 4)  # one head of width 4, 2 tokens
    c1, s1 = roformer.rope_tables(freqs, 2, 1.0)
    y = roformer.rope_apply(x, c1, s1, 1)
    t, a = 1, 1.0
    assert np.isclose(y[0, 1, 0], x[0, 1, 0] * np.cos(a) - x[0, 1, 1] * np.sin(a))
    assert np.isclose(y[0, 1, 1], x[0, 1, 1] * np.cos(a) + x[0, 1, 0] * np.sin(a))
