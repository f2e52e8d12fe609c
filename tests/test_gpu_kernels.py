"""GPU parity of the kernel plug-in API (include/ancha_b200.h) against the oracle.

Mirrors the reference's hardware contracts (tests/cuda_contracts.rs:195-401): fused and
gated attention on partial tiles, a single token and strided layouts; GEMM epilogues
(bias + GELU + residual, RoPE); custom GEMM shapes; plus the device STFT / iSTFT / OLA
against oracle/dsp.py. fp32 results must match within the reference's 1e-5.
"""
import math

import numpy as np
import pytest

from tests._util import bf16_round, max_abs, snr_db, wave

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from ancha_b200 import fused  # noqa: E402
from ancha_b200 import _native as N  # noqa: E402
from oracle import dsp, kernels, roformer  # noqa: E402


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda").to(dtype)


def oracle_attention(q, k, v):
    """[groups, tokens, heads, 64] with q pre-scaled → softmax(q kᵀ) v in float64."""
    g, t, h, d = q.shape
    qh = np.transpose(q, (0, 2, 1, 3)).reshape(g * h, t, d) * math.sqrt(d)  # dense() divides by sqrt(d)
    kh = np.transpose(k, (0, 2, 1, 3)).reshape(g * h, t, d)
    vh = np.transpose(v, (0, 2, 1, 3)).reshape(g * h, t, d)
    o = kernels.dense(qh, kh, vh, g * h, t, t, d, d).reshape(g, h, t, d)
    return np.transpose(o, (0, 2, 1, 3))


@pytest.mark.parametrize("groups,tokens,heads,strided", [
    (2, 1, 1, False), (3, 63, 2, False), (2, 65, 1, True), (1, 130, 3, False)])
def test_fused_attention_matches_oracle(groups, tokens, heads, strided):
    width = 128 if strided else 64
    inp = lambda s: wave([groups, tokens, heads, width], s)[..., :64]
    q, k, v = inp(0.1) * np.float32(0.4), inp(1.3), inp(2.9)
    qs = (q * np.float32(0.125)).astype(np.float32)
    expected = oracle_attention(qs, k, v)
    tq = dev(wave([groups, tokens, heads, width], 0.1) * np.float32(0.4 * 0.125))[..., :64]
    out = fused.attention(tq, dev(k), dev(v))
    assert max_abs(out.cpu().numpy(), expected) < 1e-5
    # Gated form over the packed q | k | v | gates | padding layout.
    gates = wave([groups, tokens, heads], 4.4) * np.float32(3.0)
    flat = lambda a: a.reshape(groups, tokens, heads * 64)
    packed = np.concatenate([flat(qs), flat(k), flat(v), gates, np.zeros((groups, tokens, 5), np.float32)], 2)
    got = fused.gated_attention(dev(packed), heads).cpu().numpy()
    gated = expected / (1.0 + np.exp(-gates.astype(np.float64)))[..., None]
    assert max_abs(got, gated) < 1e-5
    # bf16 operands: same math on the rounded inputs, bf16 output rounding.
    gotb = fused.gated_attention(dev(packed, torch.bfloat16), heads).float().cpu().numpy()
    pb = bf16_round(packed)
    qb, kb, vb = (pb[..., i * heads * 64:(i + 1) * heads * 64].reshape(groups, tokens, heads, 64) for i in range(3))
    gb = pb[..., 3 * heads * 64:3 * heads * 64 + heads]
    refb = oracle_attention(qb, kb, vb) / (1.0 + np.exp(-gb.astype(np.float64)))[..., None]
    assert max_abs(gotb, refb) < 1e-2


def test_attention_rejects_narrow_heads():
    narrow = dev(wave([1, 8, 1, 32], 0.0))
    assert fused.attention(narrow, narrow, narrow) is None


@pytest.mark.parametrize("axis", ["time", "band"])
def test_config2_attention_with_rope(axis):
    """The attention benchmark: non-causal attention with RoPE on q and k, q/k/v ~ N(0, 1).
    Time axis [B=60, H=8, T=801]; band axis [B=801, H=8, S=60] (a 40-group slice is checked)."""
    rng = np.random.default_rng(7)
    groups, tokens = (60, 801) if axis == "time" else (40, 60)
    h, d = 8, 64
    q, k, v = (rng.standard_normal((groups, tokens, h, d), dtype=np.float32) for _ in range(3))
    freqs = (10000.0 ** (-np.arange(32) / 32.0)).astype(np.float32)
    qc, qs_ = roformer.rope_tables(freqs, tokens, 1.0 / 8.0)
    kc, ks_ = roformer.rope_tables(freqs, tokens, 1.0)
    qr = roformer.rope_apply(q.reshape(groups, tokens, h * d), qc, qs_, h).reshape(groups, tokens, h, d)
    kr = roformer.rope_apply(k.reshape(groups, tokens, h * d), kc, ks_, h).reshape(groups, tokens, h, d)
    qr, kr = qr.astype(np.float32), kr.astype(np.float32)
    for dt, tol in [(torch.float32, 1e-4), (torch.bfloat16, None)]:
        got = fused.attention(dev(qr, dt), dev(kr, dt), dev(v, dt)).float().cpu().numpy()
        if dt == torch.float32:
            ref = oracle_attention(qr, kr, v)
            assert max_abs(got, ref) < tol
        else:
            ref = oracle_attention(bf16_round(qr), bf16_round(kr), bf16_round(v))
            assert snr_db(ref, got) > 45.0


def t64(a):
    return a.double().cpu().numpy()


def test_gemm_epilogues_match_reference_ops():
    # cuda_contracts.rs:253-298
    groups, tokens, k, heads = 3, 70, 64, 2
    rows, width = groups * tokens, heads * 64
    m = 3 * width
    x, w = wave([rows, k], 0.3), wave([k, m], 1.1) * np.float32(0.1)
    b, r = wave([m], 2.2), wave([rows, m], 3.3)
    projected = x.astype(np.float64) @ w.astype(np.float64) + b
    gelu = 0.5 * projected * (1.0 + np.vectorize(math.erf)(projected / math.sqrt(2.0)))
    got = fused.linear(dev(x), dev(w), fused.Epilogue(bias=dev(b), gelu=True, residual=dev(r)))
    assert max_abs(t64(got), gelu + r) < 1e-5
    freqs = (10000.0 ** (-np.arange(32) / 32.0)).astype(np.float32)
    qc, qs_ = roformer.rope_tables(freqs, tokens, 1.0 / 8.0)
    kc, ks_ = roformer.rope_tables(freqs, tokens, 1.0)
    table = np.stack([qc, qs_, kc, ks_]).astype(np.float32)
    y = projected.reshape(groups, tokens, m)
    expected = np.concatenate([roformer.rope_apply(y[..., :width], qc, qs_, heads),
                               roformer.rope_apply(y[..., width:2 * width], kc, ks_, heads),
                               y[..., 2 * width:]], 2).reshape(rows, m)
    got = fused.linear(dev(x), dev(w), fused.Epilogue(bias=dev(b), rotary=(dev(table), width)))
    assert max_abs(t64(got), expected) < 1e-5


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_linear_row_scale(dt):
    """The plug-in API's row_scale: unit_norm of the input rows applied after the product
    (roformer.rs:16-24 then the Linear), on the FFMA (f32) and tcgen05 (f16) paths."""
    rows, k, m = 300, 384, 512
    x = wave([rows, k], 0.7) * np.float32(3.0)
    w = wave([m, k], 1.9) * np.float32(0.05)
    b = wave([m], 2.5)
    inv = (1.0 / np.maximum(np.linalg.norm(x.astype(np.float64), axis=1), 1e-12)).astype(np.float32)
    td = torch.float32 if dt == "f32" else torch.float16
    xd, wd = dev(x).to(td), dev(w).to(td)
    got = t64(fused.linear(xd, wd, fused.Epilogue(bias=dev(b), gelu=True, row_scale=dev(inv)),
                           weight_layout=N.W_NK))
    xe, we = xd.double().cpu().numpy(), wd.double().cpu().numpy()
    pre = (xe @ we.T) * inv[:, None].astype(np.float64) + b
    ref = 0.5 * pre * (1.0 + np.vectorize(math.erf)(pre / math.sqrt(2.0)))
    tol = 1e-5 if dt == "f32" else 2e-3 * np.abs(ref).max()
    assert max_abs(got, ref) < tol


@pytest.mark.parametrize("rows,k,m,bias,strided", [
    (1, 8, 128, True, False), (127, 256, 256, False, False), (129, 64, 384, True, True),
    (300, 1024, 128, True, False)])
def test_custom_gemm_shapes(rows, k, m, bias, strided):
    # cuda_contracts.rs:346-374
    width = k + 16 if strided else k
    xf = wave([rows, width], 0.2)
    x = dev(xf)[:, :k]
    w = wave([k, m], 1.7) * np.float32(0.05)
    bv = wave([m], 3.1)
    expected = xf[:, :k].astype(np.float64) @ w.astype(np.float64) + (bv if bias else 0.0)
    got = fused.linear(x, dev(w), fused.Epilogue(bias=dev(bv) if bias else None))
    assert max_abs(t64(got), expected) < 1e-5
    # The same problem through the bf16 tensor-core path with PyTorch [m, k] weights.
    gotb = fused.linear(x.to(torch.bfloat16), dev(w.T.copy(), torch.bfloat16),
                        fused.Epilogue(bias=dev(bv) if bias else None), weight_layout=N.W_NK)
    refb = bf16_round(xf[:, :k]).astype(np.float64) @ bf16_round(w).astype(np.float64) + (bv if bias else 0.0)
    assert snr_db(refb, t64(gotb)) > 45.0


@pytest.mark.parametrize("rows,k,m", [(7, 8, 8), (30, 16, 24), (5, 32, 64), (4, 64, 96), (3, 8, 4)])
def test_padded_narrow_gemm(rows, k, m):
    # cuda_contracts.rs:375-384
    x, w = wave([rows, k], 0.2), wave([k, m], 1.7) * np.float32(0.05)
    got = fused.linear(dev(x), dev(w))
    assert tuple(got.shape) == (rows, m)
    assert max_abs(t64(got), x.astype(np.float64) @ w.astype(np.float64)) < 1e-5


def test_gemm_rejections():
    # cuda_contracts.rs:385-400
    x = dev(wave([4, 16], 0.0))
    assert fused.linear(x, dev(wave([16, 8], 0.0))) is not None
    assert fused.linear(x, dev(wave([16, 8], 0.0)), fused.Epilogue(bias=dev(wave([8], 0.3)))) is None
    assert fused.linear(dev(wave([4, 12], 0.0)), dev(wave([12, 128], 0.0))) is None


def stft_device(audio):
    """audio [chunks, 2, samples] → packed [chunks, frames, 4100] via the C ABI."""
    import ctypes as C
    chunks, _, samples = audio.shape
    hop = 441
    frames = samples // hop + 1
    a = dev(audio)
    out = torch.empty((chunks, frames, 4100), dtype=torch.float32, device="cuda")
    N.check(N.lib().ancha_stft_fwd(a.data_ptr(), chunks, samples, hop, out.data_ptr(), None))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("samples", [1025, 4103, 44100])
def test_stft_matches_oracle(samples):
    rng = np.random.default_rng(samples)
    audio = (rng.standard_normal((2, 2, samples)) * 0.1).astype(np.float32)
    got = stft_device(audio).cpu().numpy()
    st = dsp.Stft(2048, 441)
    for c in range(2):
        spectra = [st.forward(audio[c, ch]) for ch in range(2)]
        from oracle.runtime import pack_spectrum
        ref = pack_spectrum(spectra)
        assert max_abs(got[c], ref) < 1e-5 * np.max(np.abs(ref)) * 10


def test_stft_dc_known_answer():
    # audio_contracts.rs:38-49 with hop 441: constant 1 → bin0 = 1024, bin1 = -512.
    audio = np.ones((1, 2, 4096), np.float32)
    got = stft_device(audio).cpu().numpy()[0]
    assert abs(got[0, 0] - 1024.0) < 1e-3
    assert abs(got[0, 4] + 512.0) < 1e-3
    assert abs(got[0, 8]) < 1e-3 and abs(got[0, 9]) < 1e-3


@pytest.mark.parametrize("zero_dc", [False, True])
def test_masked_istft_matches_oracle(zero_dc):
    import ctypes as C
    from oracle.runtime import apply_masks
    rng = np.random.default_rng(3)
    samples, hop, stems, chunks = 44100, 441, 2, 2
    frames = samples // hop + 1
    audio = (rng.standard_normal((chunks, 2, samples)) * 0.1).astype(np.float32)
    packed = stft_device(audio)
    masks = (rng.standard_normal((chunks, stems, 2050, 2, frames)) * 0.5).astype(np.float32)
    dm = dev(masks)
    scratch = torch.empty(chunks * stems * 2 * frames * 2048 + 4, dtype=torch.float32, device="cuda")
    out = torch.empty((chunks, stems, 2, samples), dtype=torch.float32, device="cuda")
    N.check(N.lib().ancha_istft_masked(packed.data_ptr(), dm.data_ptr(), chunks, stems, samples, hop,
                                       int(zero_dc), scratch.data_ptr(), out.data_ptr(), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    st = dsp.Stft(2048, hop)
    pk = packed.cpu().numpy().astype(np.float64).reshape(chunks, frames, 1025, 2, 2)
    for c in range(chunks):
        spectra = [pk[c, :, :, ch, 0] + 1j * pk[c, :, :, ch, 1] for ch in range(2)]
        ref = apply_masks(spectra, masks[c].astype(np.float64), st, samples, zero_dc)
        assert max_abs(got[c], ref) < 2e-6 * max(1.0, np.max(np.abs(ref))) * 10


def test_overlap_add_matches_oracle():
    import ctypes as C
    rng = np.random.default_rng(5)
    chunk, overlap, length, planes = 4096, 4, 15000, 4
    plan = dsp.ChunkPlan(chunk, overlap)
    starts = plan.starts(length)
    y = rng.standard_normal((len(starts), planes, chunk)).astype(np.float32)
    sums = torch.zeros((planes, length), dtype=torch.float32, device="cuda")
    weights = torch.zeros(length, dtype=torch.float32, device="cuda")
    st = (C.c_int64 * len(starts))(*starts)
    dy = dev(y)
    N.check(N.lib().ancha_ola_add(dy.data_ptr(), len(starts), planes, chunk, overlap, st, length,
                                  sums.data_ptr(), weights.data_ptr(), None))
    torch.cuda.synchronize()
    acc = dsp.Accumulator(planes, length)
    for i, s in enumerate(starts):
        acc.add(plan, s, y[i])
    assert max_abs(weights.cpu().numpy(), acc.weights) < 1e-5
    assert max_abs(sums.cpu().numpy(), acc.sums) < 1e-4


def linear_abi(x, w_nk, act=N.ACT_NONE, bias=None, residual=None, rope=None, rope_width=0,
               rope_tokens=1, rope_div=1, layout=N.W_NK, out_dtype=None, workspace=False):
    """Call ancha_linear_fwd directly (ancha_linear_fwd_ws with the workspace the library asks
    for when `workspace`); w_nk is [n, k] (transposed here for W_KN)."""
    import ctypes as C
    m, k = x.shape
    n = w_nk.shape[0]
    w = w_nk if layout == N.W_NK else w_nk.t().contiguous()
    n_out = n // 2 if act == N.ACT_GLU else n
    out_dtype = out_dtype or (torch.float32 if act == N.ACT_GLU else x.dtype)
    out = torch.empty((m, n_out), dtype=out_dtype, device="cuda")
    code = {torch.float32: N.F32, torch.bfloat16: N.BF16, torch.float16: N.F16}
    d = N.LinearDesc(m, n, k, code[x.dtype], code[out_dtype], layout, x.stride(0), w.stride(0),
                     out.stride(0), residual.stride(0) if residual is not None else 0, act,
                     rope_width, rope_tokens, rope_div)
    p = lambda t: None if t is None else t.data_ptr()
    if workspace:
        nbytes = C.c_size_t(0)
        N.check(N.lib().ancha_linear_workspace(C.byref(d), C.byref(nbytes)))
        ws = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device="cuda")
        N.check(N.lib().ancha_linear_fwd_ws(C.byref(d), x.data_ptr(), w.data_ptr(), p(bias), p(residual),
                                            p(rope), out.data_ptr(), ws.data_ptr(), nbytes.value, None))
    else:
        N.check(N.lib().ancha_linear_fwd(C.byref(d), x.data_ptr(), w.data_ptr(), p(bias), p(residual),
                                         p(rope), out.data_ptr(), None))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", ["plain", "gelu", "tanh", "glu", "rope", "residual"])
@pytest.mark.parametrize("shape", [(300, 1664, 384), (48060 // 30, 1536, 384), (257, 384, 1536)])
def test_tensor_core_gemm_matches_ffma(dt, case, shape):
    """The tcgen05 kernel (NK weights) against the FFMA kernel (KN weights) on the same
    rounded operands: both accumulate in fp32, so they agree to summation order."""
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    x = torch.randn(m, k, device="cuda", generator=g).to(dt)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(dt)
    bias = torch.randn(n, device="cuda", generator=g)
    kw = dict(bias=bias)
    if case == "gelu":
        kw["act"] = N.ACT_GELU
    elif case == "tanh":
        kw["act"] = N.ACT_TANH
    elif case == "glu":
        kw["act"] = N.ACT_GLU
    elif case == "residual":
        kw["residual"] = torch.randn(m, n, device="cuda", generator=g)
        kw["out_dtype"] = torch.float32
    elif case == "rope":
        if n < 1024:
            pytest.skip("rotary columns need n >= 2·512")
        tokens = 10 if m % 10 == 0 else 1
        freqs = (10000.0 ** (-np.arange(32) / 32.0)).astype(np.float32)
        qc, qs_ = roformer.rope_tables(freqs, tokens, 1.0 / 8.0)
        kc, ks_ = roformer.rope_tables(freqs, tokens, 1.0)
        kw["rope"] = dev(np.stack([qc, qs_, kc, ks_]).astype(np.float32))
        kw.update(rope_width=512, rope_tokens=tokens, rope_div=1)
    ref = linear_abi(x, w, layout=N.W_KN, **kw).double()
    scale = ref.abs().max().item()
    # The tensor-core path with and without a workspace (the rotary table read as given, or
    # rewritten pair-major into the workspace).
    for ws in (False, True):
        tc = linear_abi(x, w, layout=N.W_NK, workspace=ws, **kw).double()
        err = (tc - ref).abs().max().item()
        # 16-bit outputs may differ by one rounding step; f32 outputs only by summation order.
        assert err <= (8e-3 if kw.get("out_dtype") is None and case != "glu" else 1e-4) * max(scale, 1.0), \
            (case, ws, err, scale)


def attention_abi(buf, desc_kw, separate_kv=False, out_dtype=None, workspace=True):
    """ancha_attention_fwd_ws (with the workspace the library asks for) or, with
    workspace=False, ancha_attention_fwd on a packed [rows, ld] buffer; separate_kv copies k / v
    into their own buffers (which routes the call to the FFMA kernel)."""
    import ctypes as C
    rows, ld = buf.shape
    heads = desc_kw["heads"]
    out = torch.zeros((rows, heads * 64), dtype=buf.dtype, device="cuda")
    code = {torch.float32: N.F32, torch.bfloat16: N.BF16, torch.float16: N.F16}[buf.dtype]
    d = N.AttnDesc(desc_kw["groups"], desc_kw["tokens"], heads, 64, code, ld, heads * 64,
                   desc_kw["group_inner"], desc_kw["inner_stride"], desc_kw["outer_stride"],
                   desc_kw["token_stride"], 0, heads * 64, 2 * heads * 64,
                   3 * heads * 64 if desc_kw.get("gated") else -1, 0)
    k = buf.clone() if separate_kv else buf
    v = buf.clone() if separate_kv else buf
    gate = buf if desc_kw.get("gated") else None
    g = None if gate is None else gate.data_ptr()
    if workspace:
        nbytes = C.c_size_t(0)
        N.check(N.lib().ancha_attention_workspace(C.byref(d), C.byref(nbytes)))
        ws = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device="cuda")
        N.check(N.lib().ancha_attention_fwd_ws(C.byref(d), buf.data_ptr(), k.data_ptr(), v.data_ptr(), g,
                                               out.data_ptr(), ws.data_ptr(), nbytes.value, None))
    else:
        N.check(N.lib().ancha_attention_fwd(C.byref(d), buf.data_ptr(), k.data_ptr(), v.data_ptr(), g,
                                            out.data_ptr(), None))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("dt,min_db", [(torch.float16, 60.0), (torch.bfloat16, 45.0)])
@pytest.mark.parametrize("axis", ["time", "band", "band2", "short", "t129", "t200", "t300"])
@pytest.mark.parametrize("gated", [False, True])
def test_tensor_core_attention_matches_ffma(dt, min_db, axis, gated):
    """The tcgen05 attention against the FFMA attention on the same 16-bit operands, in the
    model's layouts: time axis (60 bands × 801 frames, tokens contiguous), band axis (801
    frames × 60 bands, tokens 801 rows apart, two problems per tile; and two chunks of 51
    frames × 33 bands, so the last tile of each chunk holds one problem), a short ragged case,
    and time axes whose last key block holds 1, 33, 44 (at most 64: S computed for 64 keys) or
    72 valid keys."""
    chunks, bands, frames, heads = {"time": (1, 60, 801, 8), "band": (1, 60, 801, 8), "band2": (2, 33, 51, 3),
                                     "short": (2, 3, 37, 2), "t129": (1, 4, 129, 2),
                                     "t200": (1, 3, 200, 2), "t300": (2, 3, 300, 2)}[axis]
    ld = (3 * heads * 64 + heads + 7) // 8 * 8   # 16-byte rows, as the model's packed projection
    rows = chunks * bands * frames
    g = torch.Generator(device="cuda").manual_seed(5)
    buf = (torch.randn(rows, ld, device="cuda", generator=g) * 0.7).to(dt)
    if not axis.startswith("band"):
        kw = dict(groups=chunks * bands, tokens=frames, group_inner=chunks * bands, inner_stride=frames,
                  outer_stride=0, token_stride=1)
    else:
        kw = dict(groups=chunks * frames, tokens=bands, group_inner=frames, inner_stride=1,
                  outer_stride=bands * frames, token_stride=frames)
    kw.update(heads=heads, gated=gated)
    tc = attention_abi(buf, kw).double().cpu().numpy()
    ref = attention_abi(buf, kw, separate_kv=True).double().cpu().numpy()
    snr = snr_db(ref, tc)
    print(f"attention tc vs ffma {axis} {dt} gated={gated}: {snr:.1f} dB")
    assert np.all(np.isfinite(tc)) and np.abs(ref).max() > 0 and snr >= min_db
    assert snr < 200.0  # the two kernels really differ (P is rounded to 16 bits on the tensor path)


@pytest.mark.parametrize("axis", ["time", "t129", "t200", "t300", "band", "band2"])
@pytest.mark.parametrize("gated", [False, True])
def test_fp32_split_attention_matches_ffma(axis, gated):
    """fp32 attention on the tensor cores (q, k, v split into three bf16 planes, six plane
    products for S and for P·V, P split in the softmax) against the FFMA attention on the same
    f32 operands, which is held to the oracle at 1e-5, and against float64: the time axis of the
    model (60 bands × 801 frames), time axes whose last key block holds 1, 72 or 44 valid keys,
    and the band axis (801 frames × 60 bands, tokens 801 rows apart; two chunks of 51 frames ×
    33 bands)."""
    chunks, bands, frames, heads = {"time": (1, 60, 801, 8), "t129": (1, 4, 129, 2), "t200": (1, 3, 200, 2),
                                    "t300": (2, 3, 300, 2), "band": (1, 60, 801, 8),
                                    "band2": (2, 33, 51, 3)}[axis]
    ld = (3 * heads * 64 + heads + 7) // 8 * 8
    rows = chunks * bands * frames
    g = torch.Generator(device="cuda").manual_seed(11)
    buf = torch.randn(rows, ld, device="cuda", generator=g) * 0.7
    if not axis.startswith("band"):
        kw = dict(groups=chunks * bands, tokens=frames, group_inner=chunks * bands, inner_stride=frames,
                  outer_stride=0, token_stride=1)
    else:
        kw = dict(groups=chunks * frames, tokens=bands, group_inner=frames, inner_stride=1,
                  outer_stride=bands * frames, token_stride=frames)
    kw.update(heads=heads, gated=gated)
    tc = attention_abi(buf, kw).double().cpu().numpy()
    ffma = attention_abi(buf, kw, separate_kv=True).double().cpu().numpy()
    # Without a workspace the same call runs the FFMA kernel (no allocation inside the call).
    plain = attention_abi(buf, kw, workspace=False).double().cpu().numpy()
    assert np.array_equal(plain, ffma)
    # float64 attention of the first (up to) four groups from the same f32 operands
    b = buf.double().cpu().numpy()
    tokens = kw["tokens"]
    got_tc, got_ffma, exact = [], [], []
    for gi in range(min(4, kw["groups"])):
        r0 = (gi // kw["group_inner"]) * kw["outer_stride"] + (gi % kw["group_inner"]) * kw["inner_stride"]
        r = r0 + np.arange(tokens) * kw["token_stride"]
        for h in range(heads):
            q, k, v = (b[r, c + h * 64:c + (h + 1) * 64] for c in (0, heads * 64, 2 * heads * 64))
            sc = q @ k.T
            pr = np.exp(sc - sc.max(axis=1, keepdims=True))
            o = (pr / pr.sum(axis=1, keepdims=True)) @ v
            if gated:
                o = o / (1.0 + np.exp(-b[r, 3 * heads * 64 + h]))[:, None]
            exact.append(o)
            got_tc.append(tc[r, h * 64:(h + 1) * 64])
            got_ffma.append(ffma[r, h * 64:(h + 1) * 64])
    exact, got_tc, got_ffma = np.stack(exact), np.stack(got_tc), np.stack(got_ffma)
    e_tc, e_ffma = np.abs(got_tc - exact).max(), np.abs(got_ffma - exact).max()
    scale = np.abs(exact).max()
    snr = snr_db(ffma, tc)
    print(f"fp32 split attention {axis} gated={gated}: vs float64 max abs {e_tc:.2e}, FFMA vs float64 "
          f"{e_ffma:.2e} (|o| ≤ {scale:.2f}); split vs FFMA {snr:.1f} dB")
    assert np.all(np.isfinite(tc)) and scale > 0
    assert e_tc <= 1e-5 * max(scale, 1.0) and snr >= 100.0
