"""Kernel microbenchmarks: fused attention and the projection GEMMs in isolation.

The counterpart of the reference's CUDA examples ``crates/ancha-models/examples/
fused_attention.rs`` (fused vs materialised attention, 13-75) and ``fused_linear.rs``
(custom GEMM vs Burn matmul, 7-55), on this library's kernels. Shapes are the Mel-Band
RoFormer's at one 8 s chunk (60 bands × 801 frames, dim 384, 8 × 64 heads) and the attention
benchmark's (time axis [B=60, H=8, T, 64] for T ∈ {801, 1601, 3201}; band axis
[B=801, H=8, S=60, 64]). Times are CUDA-event averages after warm-up; FLOPs are algorithmic
(attention 4·B·H·T²·D, GEMM 2·M·N·K with unpadded N).

    python -m ancha_b200.microbench [--kernel all|gemm|attention|mdx23c|mdxnet] [--reps N] [--dtype f16]
"""
from __future__ import annotations

import argparse
import json


def _time(fn, reps, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def gemm_cases(rows=60 * 801):
    """(name, m, n, k, epilogue kind) of every projection of one Mel chunk."""
    return [("qkv_gate_rope", rows, 1544, 384, "rope"), ("attn_out_residual", rows, 384, 512, "residual"),
            ("ffn_in_gelu", rows, 1536, 384, "gelu"), ("ffn_out_residual", rows, 384, 1536, "residual"),
            ("mask_hidden1_tanh", rows, 1536, 384, "tanh"), ("mask_hidden2_tanh", rows, 1536, 1536, "tanh")]


def run_gemm(dtype, reps):
    import torch
    from . import _native as N
    from .fused import Epilogue, linear
    out = []
    for name, m, n, k, kind in gemm_cases():
        x = torch.randn(m, k, device="cuda").to(dtype)
        w = (torch.randn(n, k, device="cuda") * 0.02).to(dtype)
        ep = Epilogue(bias=torch.zeros(n, device="cuda"))
        if kind == "gelu":
            ep.gelu = True
        elif kind == "residual":
            ep = Epilogue(residual=torch.randn(m, n, device="cuda"))
        if kind == "tanh":
            fn = _abi_linear(x, w, N.ACT_TANH)
        elif kind == "rope":
            # n = 1544 is not a multiple of 128, where fused.linear returns the reference's None;
            # the model calls the ABI directly with the rotary table.
            tab = torch.zeros(4, 801, 64, device="cuda")
            tab[0] = tab[2] = 1.0
            fn = _abi_linear(x, w, N.ACT_NONE, rope=tab)
        else:
            fn = (lambda x=x, w=w, ep=ep: linear(x, w, ep, weight_layout=N.W_NK))
        ms = _time(fn, reps)
        tf = 2.0 * m * n * k / (ms / 1e3) / 1e12
        out.append({"kernel": "gemm_tc", "case": name, "m": m, "n": n, "k": k, "ms": ms, "tflops": tf})
    return out


def _abi_linear(x, w, act, rope=None):
    """ancha_linear_fwd_ws with NK weights, a bias and the workspace the library asks for (the
    RoPE epilogue when given)."""
    import ctypes as C

    import torch
    from . import _native as N
    m, k = x.shape
    n = w.shape[0]
    y = torch.empty(m, n, dtype=x.dtype, device="cuda")
    b = torch.zeros(n, device="cuda")
    code = N.BF16 if x.dtype == torch.bfloat16 else N.F16
    tokens = rope.shape[1] if rope is not None else 1
    d = N.LinearDesc(m, n, k, code, code, N.W_NK, k, k, n, 0, act, 512 if rope is not None else 0, tokens, 1)
    rp = None if rope is None else rope.data_ptr()
    nbytes = C.c_size_t(0)
    N.check(N.lib().ancha_linear_workspace(C.byref(d), C.byref(nbytes)))
    ws = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device="cuda")
    return lambda: N.check(N.lib().ancha_linear_fwd_ws(C.byref(d), x.data_ptr(), w.data_ptr(), b.data_ptr(),
                                                       None, rp, y.data_ptr(), ws.data_ptr(), nbytes.value, None))


def run_attention(dtype, reps):
    import torch
    from .fused import attention, gated_attention
    out = []
    for t in (801, 1601, 3201):
        q = torch.randn(60, t, 8, 64, device="cuda").to(dtype)
        ms = _time(lambda q=q: attention(q, q, q), reps)
        flops = 4.0 * 60 * 8 * t * t * 64
        out.append({"kernel": "attention_tc", "case": f"time_T{t}", "ms": ms, "tflops": flops / (ms / 1e3) / 1e12})
    # Band axis inside the model layout: 801 frames × 8 heads, 60 tokens T rows apart.
    import ctypes as C
    from . import _native as N
    rows, ld = 60 * 801, 1544
    buf = torch.randn(rows, ld, device="cuda").to(dtype)
    o = torch.empty(rows, 512, device="cuda", dtype=dtype)
    code = N.BF16 if dtype == torch.bfloat16 else N.F16
    d = N.AttnDesc(801, 60, 8, 64, code, ld, 512, 801, 1, 0, 801, 0, 512, 1024, 1536, 0)
    fn = lambda: N.check(N.lib().ancha_attention_fwd(C.byref(d), buf.data_ptr(), buf.data_ptr(), buf.data_ptr(),
                                                     buf.data_ptr(), o.data_ptr(), None))
    ms = _time(fn, reps)
    flops = 4.0 * 801 * 8 * 60 * 60 * 64
    moved = rows * (3 * 512 + 8) * 2 + rows * 512 * 2
    out.append({"kernel": "attention_tc", "case": "band_S60_gated", "ms": ms, "tflops": flops / (ms / 1e3) / 1e12,
                "gbs": moved / (ms / 1e3) / 1e9})
    return out


def run_mdx23c(dtype_name, reps):
    """MDX23C inst_voc_hq2 forward (the benchmarked network, synthetic seeded weights) on
    one chunk: [1, 4, 4096, 256] → [1, 8, 4096, 256]."""
    import shutil
    import tempfile

    import torch

    from .mdx23c import Mdx23c, forward_flops, inst_voc_hq2, random_tensors, write_package
    c = inst_voc_hq2()
    d = tempfile.mkdtemp(prefix="mdx23c-bench-")
    try:
        write_package(d, c, random_tensors(c))
        m = Mdx23c(d, 0, dtype_name)
    finally:
        shutil.rmtree(d, ignore_errors=True)
    x = torch.randn(1, 4, c["bins"], c["frames"], device="cuda")
    ms = _time(lambda: m.forward(x), reps)
    flops = forward_flops(c, 1, c["frames"])
    step_s = c["hop"] * (c["frames"] - 1) / c["overlap"] / c["sample_rate"]  # new audio per chunk
    return [{"kernel": "mdx23c_forward", "case": "inst_voc_hq2 batch 1 frames 256", "dtype": dtype_name,
             "ms": ms, "tflops": flops / (ms / 1e3) / 1e12, "x_realtime_model_only": step_s / (ms / 1e3)}]


def run_mdxnet(dtype_name, reps):
    """BASELINE config 5's synthetic classic MDX-Net (TFC-TDF v1 ONNX graph, n_fft 6144, dim_f
    3072, dim_t 256) through the classic MDX executor with conv_gemm in ``dtype_name``: one call of
    batch 4, [4, 4, 3072, 256]."""
    import torch

    from .mdx import Graph
    from .mdx_net import MdxNetConfig, forward_flops, tfc_tdf_v1
    c = MdxNetConfig()
    g = Graph(tfc_tdf_v1(c, seed=0), 0, True, gemm=dtype_name)
    x = torch.randn(4, 4, c.dim_f, c.dim_t, device="cuda") * 0.1
    ms = _time(lambda: g.forward(x), reps, warmup=2)
    g.close()
    return [{"kernel": "mdx_graph_forward", "case": "tfc-tdf v1 batch 4", "dtype": dtype_name, "ms": ms,
             "tflops": forward_flops(c, 4) / (ms / 1e3) / 1e12}]


def main(argv=None):
    import torch
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--kernel", default="all", choices=["all", "gemm", "attention", "mdx23c", "mdxnet"])
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--dtype", default="f16", choices=["f16", "bf16", "f32"])
    a = p.parse_args(argv)
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[a.dtype]
    res = []
    if a.kernel in ("all", "gemm"):
        res += run_gemm(dt, a.reps)
    if a.kernel in ("all", "attention"):
        res += run_attention(dt, a.reps)
    if a.kernel == "mdx23c":
        res += run_mdx23c(a.dtype, a.reps)
    if a.kernel == "mdxnet":
        res += run_mdxnet(a.dtype, a.reps)
    for r in res:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
