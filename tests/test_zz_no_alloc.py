"""ancha_istft_masked_static (library-owned scratch, no allocation) against ancha_istft_masked.

Both entry points run the same frame and overlap kernels; the static one feeds them through
its fixed device scratch one chunk and as many stems as fit at a time. The comparison runs
two calls in a row with different masks (the second call reuses the scratch the first left
behind): with several stems in one batch, with a partial last batch of stems (15 + 2 per
chunk, which checks the mask and output offsets of the second batch and of the second chunk),
and at the Mel chunk size where each batch holds a single stem. The file name keeps it last in
collection so it also runs after every other GPU test; it needs nothing from them.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from ancha_b200 import _native as N  # noqa: E402


def _spectrum(rng, chunks, samples, hop):
    audio = torch.from_numpy((rng.standard_normal((chunks, 2, samples)) * 0.1).astype(np.float32)).cuda()
    frames = samples // hop + 1
    packed = torch.empty((chunks, frames, 1025 * 4), dtype=torch.float32, device="cuda")
    N.check(N.lib().ancha_stft_fwd(audio.data_ptr(), chunks, samples, hop, packed.data_ptr(), None))
    return packed


def _with_caller_scratch(packed, masks, chunks, stems, samples, hop, zero_dc):
    frames = samples // hop + 1
    scratch = torch.empty(chunks * stems * 2 * frames * 2048 + 4, dtype=torch.float32, device="cuda")
    out = torch.empty((chunks, stems, 2, samples), dtype=torch.float32, device="cuda")
    N.check(N.lib().ancha_istft_masked(packed.data_ptr(), masks.data_ptr(), chunks, stems, samples, hop,
                                       zero_dc, scratch.data_ptr(), out.data_ptr(), None))
    status = scratch[chunks * stems * 2 * frames * 2048:].view(torch.int32)[0]
    return out, int(status.item())


@pytest.mark.parametrize("chunks,stems,samples,hop,zero_dc",
                         [(3, 4, 44100, 441, 0),     # 101 frames: all 4 stems in one batch
                          (2, 17, 44100, 441, 1),    # 15 + 2 stems per chunk: a partial second batch
                          (2, 2, 352800, 441, 1)])   # Mel chunk, 801 frames: one stem per batch
def test_static_scratch_matches_caller_scratch(chunks, stems, samples, hop, zero_dc):
    rng = np.random.default_rng(11)
    packed = _spectrum(rng, chunks, samples, hop)
    frames = samples // hop + 1
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for call in range(2):
        masks = torch.from_numpy((rng.standard_normal((chunks, stems, 2050, 2, frames)) * 0.5)
                                 .astype(np.float32)).cuda()
        out = torch.full((chunks, stems, 2, samples), float("nan"), dtype=torch.float32, device="cuda")
        N.check(N.lib().ancha_istft_masked_static(packed.data_ptr(), masks.data_ptr(), chunks, stems,
                                                  samples, hop, zero_dc, out.data_ptr(), status.data_ptr(),
                                                  None))
        want, want_status = _with_caller_scratch(packed, masks, chunks, stems, samples, hop, zero_dc)
        torch.cuda.synchronize()
        scale = float(want.abs().max())
        err = float((out - want).abs().max())
        assert err <= 1e-6 * max(1.0, scale), f"call {call}: max |diff| {err} (scale {scale})"
        assert int(status.item()) == want_status == 0


def test_static_scratch_rejects_oversized_chunks():
    samples, hop = 1537 * 441, 441  # 1538 frames > 1536
    rng = np.random.default_rng(12)
    packed = _spectrum(rng, 1, samples, hop)
    masks = torch.zeros(1, dtype=torch.float32, device="cuda")  # never read: rejected up front
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    rc = N.lib().ancha_istft_masked_static(packed.data_ptr(), masks.data_ptr(), 1, 1, samples, hop, 0,
                                           out.data_ptr(), None, None)
    assert rc == N.E_INVALID
    msg = N.lib().ancha_last_error().decode()
    assert "1538" in msg and "1536" in msg
