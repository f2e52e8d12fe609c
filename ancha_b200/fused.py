"""Kernel plug-in API over torch CUDA tensors, mirroring the reference's ``fused`` module.

``crates/ancha-models/src/fused/mod.rs`` exposes ``attention``, ``gated_attention``,
``linear`` (+ ``Epilogue``) and ``available``; each returns ``None`` when the shape or
backend is not handled. The same functions here take CUDA tensors, call the C ABI on the
current torch stream and return ``None`` exactly where the reference does. Torch is only
the device-memory plumbing; the arithmetic runs in this library's kernels.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import ctypes as C

from . import _native as N

ATTENTION_HEAD_DIM = 64


def _torch():
    import torch
    return torch


def available(device: int = 0) -> bool:
    """Whether ``device`` is an sm_100 GPU with this library (``fused::available``)."""
    try:
        return bool(N.lib().ancha_available(device))
    except N.AnchaError:
        return False


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float32:
        return N.F32
    if t.dtype == torch.bfloat16:
        return N.BF16
    if t.dtype == torch.float16:
        return N.F16
    raise N.AnchaError(N.E_INVALID, f"unsupported dtype {t.dtype}")


def _stream():
    torch = _torch()
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _rows_view(t, name: str):
    """Row stride (elements) of a tensor whose last axis is dense."""
    if t.stride(-1) != 1:
        raise N.AnchaError(N.E_INVALID, f"{name}: last axis must be contiguous")
    return t.stride(-2) if t.dim() >= 2 else t.shape[-1]


def _workspace(query, desc, device):
    """A device workspace of the size the library asks for ``desc`` (the caller's allocation,
    through torch's caching allocator), or ``(None, 0)`` when none helps."""
    torch = _torch()
    n = C.c_size_t(0)
    N.check(query(C.byref(desc), C.byref(n)))
    if n.value == 0:
        return None, 0
    buf = torch.empty(n.value, dtype=torch.uint8, device=device)
    return buf, n.value


def attention(q, k, v):
    """``softmax(q·kᵀ)·v`` over ``[groups, tokens, heads, 64]`` with ``q`` pre-scaled
    (fused/mod.rs:20-41). Returns ``None`` unless the head width is 64 and shapes match."""
    if q.shape[-1] != ATTENTION_HEAD_DIM or k.shape != q.shape or v.shape != q.shape:
        return None
    torch = _torch()
    groups, tokens, heads, _ = q.shape
    out = torch.empty((groups, tokens, heads, 64), dtype=q.dtype, device=q.device)
    flat = [t.reshape(groups, tokens, heads * 64) if t.is_contiguous() else
            t.contiguous().reshape(groups, tokens, heads * 64) for t in (q, k, v)]
    if len({t.stride(1) for t in flat}) != 1 or any(t.stride(0) != tokens * t.stride(1) for t in flat):
        flat = [t.contiguous() for t in flat]
    d = N.AttnDesc(groups, tokens, heads, 64, _dtype_code(q), heads * 64, heads * 64, groups,
                   tokens, 0, 1, 0, 0, 0, -1, 0)
    L = N.lib()
    ws, nbytes = _workspace(L.ancha_attention_workspace, d, q.device)
    N.check(L.ancha_attention_fwd_ws(C.byref(d), flat[0].data_ptr(), flat[1].data_ptr(), flat[2].data_ptr(),
                                     None, out.data_ptr(), None if ws is None else ws.data_ptr(), nbytes,
                                     _stream()))
    return out


def gated_attention(packed, heads: int):
    """RoFormer attention core from one packed ``[groups, tokens, columns]`` projection holding
    q | k | v (``heads·64`` columns each) and the per-head gate logits after them
    (fused/mod.rs:43-55). Returns ``[groups, tokens, heads, 64]`` or ``None``."""
    if packed.shape[2] < heads * (3 * ATTENTION_HEAD_DIM + 1):
        return None
    torch = _torch()
    groups, tokens, cols = packed.shape
    p = packed if packed.stride(2) == 1 and packed.stride(0) == tokens * packed.stride(1) \
        else packed.contiguous()
    ld = p.stride(1)
    inner = heads * 64
    out = torch.empty((groups, tokens, heads, 64), dtype=packed.dtype, device=packed.device)
    d = N.AttnDesc(groups, tokens, heads, 64, _dtype_code(p), ld, inner, groups, tokens, 0, 1,
                   0, inner, 2 * inner, 3 * inner, 0)
    ptr = p.data_ptr()
    L = N.lib()
    ws, nbytes = _workspace(L.ancha_attention_workspace, d, packed.device)
    N.check(L.ancha_attention_fwd_ws(C.byref(d), ptr, ptr, ptr, ptr, out.data_ptr(),
                                     None if ws is None else ws.data_ptr(), nbytes, _stream()))
    return out


@dataclass
class Epilogue:
    """Work fused into the output pass of :func:`linear`, applied in field order
    (fused/mod.rs:57-79): bias ``[m]``, erf-GELU, interleaved RoPE (``(table [4, tokens, 64],
    width)``), residual ``[n, m]``. ``row_scale`` ``[n]`` (this engine's addition, before the
    bias) multiplies each row of the product, e.g. by 1 / ‖x_row‖ so a unit norm of the input
    rows needs no separate pass."""
    bias: Optional[object] = None
    gelu: bool = False
    rotary: Optional[tuple] = None
    residual: Optional[object] = None
    row_scale: Optional[object] = None


def linear_supported(k: int, m: int) -> bool:
    """The reference's ``linear_supported`` (fused/mod.rs:81-85)."""
    return k > 0 and k % 8 == 0 and m > 0 and m % 128 == 0


def linear(x, weight, epilogue: Epilogue = Epilogue(), weight_layout: int = N.W_KN):
    """``x [n, k] · weight [k, m]`` (Burn layout) then the epilogue (fused/mod.rs:94-176).

    Returns ``None`` where the reference does: ``k % 8 != 0``, an epilogue with ``m`` not a
    multiple of 128, or a rotary / residual operand of the wrong shape. ``weight_layout =
    W_NK`` takes a PyTorch ``[m, k]`` weight instead (the layout of the tcgen05 path).
    """
    torch = _torch()
    n, k = x.shape
    if weight_layout == N.W_KN:
        rows, m = weight.shape
    else:
        m, rows = weight.shape
    if rows != k or k == 0 or k % 8 or m == 0:
        return None
    empty = epilogue.bias is None and not epilogue.gelu and epilogue.rotary is None \
        and epilogue.residual is None and epilogue.row_scale is None
    if m % 128 and not empty:
        return None
    rope, width, tokens = None, 0, 1
    if epilogue.rotary is not None:
        table, width = epilogue.rotary
        four, tokens, dim = table.shape
        if four != 4 or dim != 64 or n % tokens or width % 64 or 2 * width > m:
            return None
        rope = table.contiguous().float()
    if epilogue.residual is not None and tuple(epilogue.residual.shape) != (n, m):
        return None
    if epilogue.row_scale is not None and tuple(epilogue.row_scale.shape) != (n,):
        return None
    xs = x if x.stride(-1) == 1 else x.contiguous()
    ws = weight if weight.stride(-1) == 1 else weight.contiguous()
    out = torch.empty((n, m), dtype=torch.float32 if x.dtype == torch.float32 else x.dtype,
                      device=x.device)
    res = epilogue.residual
    if res is not None:
        res = res.float()
        res = res if res.stride(-1) == 1 else res.contiguous()
    bias = None if epilogue.bias is None else epilogue.bias.float().contiguous()
    rs = None if epilogue.row_scale is None else epilogue.row_scale.float().contiguous()
    d = N.LinearDesc(n, m, k, _dtype_code(xs), _dtype_code(out), weight_layout,
                     xs.stride(0), ws.stride(0), m, res.stride(0) if res is not None else 0,
                     N.ACT_GELU if epilogue.gelu else N.ACT_NONE, width, tokens, 1,
                     None if rs is None else rs.data_ptr())
    ptr = lambda t: None if t is None else t.data_ptr()
    L = N.lib()
    wk, nbytes = _workspace(L.ancha_linear_workspace, d, x.device)
    N.check(L.ancha_linear_fwd_ws(C.byref(d), xs.data_ptr(), ws.data_ptr(), ptr(bias), ptr(res), ptr(rope),
                                  out.data_ptr(), ptr(wk), nbytes, _stream()))
    return out
