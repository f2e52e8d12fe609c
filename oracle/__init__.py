"""CPU oracle for the RoFormer separation path: TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference CPU path of 3tic-project/Ancha for the
Mel-Band / BS-RoFormer hot path, so that the CUDA kernels of ``ancha_b200`` can be checked
against it. It is never part of the product: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and
only as the checker or the timed CPU baseline.

Modules and the reference code each follows (paths inside the reference project):

* ``dsp``       -- ``crates/ancha-audio/src/dsp.rs`` (STFT / iSTFT / reflect padding) and
                   ``crates/ancha-audio/src/chunk.rs`` (chunk plan, linear-fade overlap-add).
* ``kernels``   -- ``crates/ancha-kernels/src/attention.rs`` (dense / online-softmax
                   attention) and ``crates/ancha-kernels/src/fusion.rs`` (norm, packing, mask).
* ``roformer``  -- ``crates/ancha-models/src/network.rs`` and ``roformer.rs`` (band split,
                   axial transformers, mask estimators) with the load-time folding of
                   ``weights.rs::folded_linear``.
* ``runtime``   -- ``src/runtime.rs`` (chunk gather, packing, complex mask, OLA, residual).

Pinning. The DSP, attention, norm, complex-mask and OLA pieces are pinned by the known
answers and invariants that the reference's own tests hold
(``crates/ancha-audio/tests/audio_contracts.rs``, ``crates/ancha-kernels/tests/contracts.rs``,
``crates/ancha-models/tests/model_contracts.rs``); ``tests/test_oracle_kat.py`` replays them.
The reference ships no golden output for any RoFormer model (its RoFormer parity is pinned
only by cross-backend equality and an MSST script that needs the network), and its Rust
toolchain is absent here, so the END-TO-END RoFormer forward is "parity unpinned": it is a
line-by-line restatement whose components are pinned, not a replay of reference outputs.

Arithmetic runs in float64 by default (``dtype=np.float32`` mirrors the reference's f32
storage). Band-group reordering in ``network.rs`` only changes the order of independent
per-band work, so the oracle runs bands in band order; the overlapping-band scatter-add is
a sum of at most two terms per bin in the Mel table.
"""
