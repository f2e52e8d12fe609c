"""MDX23C host logic without a GPU: package manifests are checked (strict keys, the
Config::validate limits of mdx23c.rs:76-122) before any device work, through the C ABI."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from ancha_b200 import _native as N
from ancha_b200.mdx23c import write_package
from oracle import mdx23c as M

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "mdx23c_tiny.json")


def _load(path):
    h = C.c_void_p()
    st = N.lib().ancha_mdx23c_load(path.encode(), 0, N.PRECISION_F32, C.byref(h))
    if st == N.OK:
        N.lib().ancha_mdx23c_free(h)
    return st, N.last_error()


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


def _package(tmp_path, golden, change=None, extra_key=False):
    c = dict(golden["config"])
    if change:
        c.update(change)
    tensors = M.fixture_weights([(w["name"], w["shape"]) for w in golden["weights"]])
    d = str(tmp_path / "pkg")
    m = write_package(d, c, tensors)
    if extra_key:
        m["config"]["unknown"] = 1
        with open(os.path.join(d, "manifest.json"), "w") as fh:
            json.dump(m, fh)
    return d


@pytest.mark.parametrize("change,message", [
    ({"frames": 7}, "encoder scales"),
    ({"bins": 31}, "encoder scales"),
    ({"scales": 0}, "2x2 down/up sampling"),
    ({"overlap": 0}, "context"),
    ({"bottleneck_factor": 0}, "network size"),
    ({"stems": ["instrumental", "vocals"]}, "vocals/instrumental"),
    ({"sample_rate": 48000}, "44100"),
    ({"frames": 2**32 + 256}, "integer out of range"),  # not read as 256 after truncation
    ({"n_fft": 1e300}, "expected an integer"),
])
def test_invalid_config_rejected_before_device_work(tmp_path, golden, change, message):
    st, err = _load(_package(tmp_path, golden, change))
    assert st == N.E_INVALID
    assert message in err


def test_unknown_manifest_field_rejected(tmp_path, golden):
    st, err = _load(_package(tmp_path, golden, extra_key=True))
    assert st == N.E_INVALID and "unknown field" in err


def test_missing_package_is_an_io_error(tmp_path):
    st, _ = _load(str(tmp_path / "absent"))
    assert st == N.E_IO


def test_forward_rejects_null_handle():
    assert N.lib().ancha_mdx23c_forward(None, None, 1, 8, None, None, None) == N.E_INVALID


def test_overlap_plan_matches_reference_and_oracle():
    # mdx23c_runtime_contracts.rs:16-24 and the oracle's restatement, through the C ABI.
    from ancha_b200.mdx23c import OverlapPlan
    p = OverlapPlan(132300, 261120, 8)
    assert (p.step, p.border, p.pad, p.chunks) == (32640, 228480, 30900, 12)
    for n in [1, 32, 127, 128, 129, 256, 333, 44100 * 37]:
        for chunk, overlap in [(128, 1), (128, 2), (128, 8), (261120, 8), (1792, 4)]:
            a, b = OverlapPlan(n, chunk, overlap), M.OverlapPlan(n, chunk, overlap)
            assert (a.step, a.border, a.pad, a.padded, a.chunks) == (b.step, b.border, b.pad, b.padded, b.chunks)
            assert [a.intersects(i * a.step) for i in range(a.chunks)] == \
                   [b.intersects(i * b.step) for i in range(b.chunks)]
    for bad in [(0, 128, 8), (10, 128, 0), (10, 128, 17), (10, 4, 8)]:
        with pytest.raises(N.AnchaError):
            OverlapPlan(*bad)
