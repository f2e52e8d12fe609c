"""Failure detection on the device, without a GPU fault: the bounded waits of the tensor-core
kernels give up after their budget, record the timeout in the library's device error word and
return, and the context stays usable (the reference covers device failures in
src/device.rs:11-41 and tests/cuda_device_failure.rs).

ancha_wait_selftest runs that wait with a short budget on an mbarrier nothing arrives at; the
call must report ANCHA_E_TIMEOUT, and the next tensor-core calls must succeed with correct results.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from ancha_b200 import _native as N  # noqa: E402
from ancha_b200 import fused  # noqa: E402


@pytest.mark.parametrize("budget", [0, 20000, 2000000])
def test_expired_wait_reports_timeout_and_the_device_stays_usable(budget):
    rc = N.lib().ancha_wait_selftest(budget, None)
    assert rc == N.E_TIMEOUT
    assert "bounded device-side wait" in N.lib().ancha_last_error().decode()
    # The error word is cleared: a tensor-core GEMM and attention run and are correct.
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(256, 128, device="cuda", generator=g).half()
    w = torch.randn(384, 128, device="cuda", generator=g).half()
    y = fused.linear(x, w, fused.Epilogue(), weight_layout=N.W_NK)
    ref = x.float() @ w.float().T
    assert float((y.float() - ref).abs().max()) <= 2e-3 * float(ref.abs().max())
    q = torch.randn(2, 200, 8, 64, device="cuda", generator=g).half() * 0.3
    o = fused.attention(q, q, q).double()
    s = torch.einsum("gqhd,gkhd->ghqk", q.double(), q.double())
    ref = torch.einsum("ghqk,gkhd->gqhd", torch.softmax(s, -1), q.double())
    assert float((o - ref).abs().max()) <= 5e-3 * float(ref.abs().max())


def test_budget_outside_the_kernel_budget_is_rejected():
    assert N.lib().ancha_wait_selftest(-1, None) == N.E_INVALID
    assert N.lib().ancha_wait_selftest(1 << 40, None) == N.E_INVALID
