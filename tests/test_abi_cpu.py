"""The C-ABI library without a GPU: it loads, exports every symbol the header declares, and
fails with a status (not a crash) when no GPU is present. No compute call runs here."""
import ctypes as C
import os
import re

import pytest

from ancha_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "ancha_b200.h")).read()
    return sorted(set(re.findall(r"ANCHA_API\s+[\w\s\*]+?\b(ancha_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    declared = header_functions()
    assert declared == sorted(N.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name


def test_exported_symbols_are_exactly_the_header():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    syms = sorted(l.split()[-1] for l in out.stdout.splitlines() if " T " in l and "ancha_" in l)
    assert syms == header_functions()


def test_version_and_status_without_gpu():
    lib = N.lib()
    assert b"sm_100a" in lib.ancha_version()
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert lib.ancha_available(0) == 0
    assert N.last_error()


def test_struct_layouts_match_header():
    # The ctypes mirrors must match the C layout (sizes of the packed descriptors).
    assert C.sizeof(N.AttnDesc) == 5 * 4 + 4 + 6 * 8 + 5 * 4 + 4  # + padding to 8
    assert C.sizeof(N.LinearDesc) == 6 * 4 + 4 * 8 + 4 * 4 + 8
    assert C.sizeof(N.SeparateOpts) == 3 * 8 + 8 + 4 * 4 + 2 * 8


def test_struct_layouts_match_the_c_compiler(tmp_path):
    """Sizes and field offsets of the descriptors as gcc lays out include/ancha_b200.h."""
    import shutil
    import subprocess
    if not shutil.which("gcc"):
        pytest.skip("no gcc")
    structs = {"ancha_attn_desc": N.AttnDesc, "ancha_linear_desc": N.LinearDesc,
               "ancha_separate_opts": N.SeparateOpts}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "ancha_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'printf("{cname}.{field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(got[cname]) == C.sizeof(py), cname
        for field, _ in py._fields_:
            assert int(got[f"{cname}.{field}"]) == getattr(py, field).offset, f"{cname}.{field}"


def test_workspace_queries():
    """The workspace variants say how many bytes help (pure host arithmetic, no GPU)."""
    lib = N.lib()
    n = C.c_size_t(7)
    # f32 time axis over a packed [60 · 801, 1544] buffer: three bf16 planes of the used
    # 3 · 512 q | k | v columns of all 48 060 rows.
    d = N.AttnDesc(60, 801, 8, 64, N.F32, 1544, 512, 60, 801, 0, 1, 0, 512, 1024, 1536, 0)
    assert lib.ancha_attention_workspace(C.byref(d), C.byref(n)) == N.OK
    assert n.value == 3 * 60 * 801 * 1536 * 2
    d16 = N.AttnDesc(60, 801, 8, 64, N.F16, 1544, 512, 60, 801, 0, 1, 0, 512, 1024, 1536, 0)
    assert lib.ancha_attention_workspace(C.byref(d16), C.byref(n)) == N.OK and n.value == 0
    ld = N.LinearDesc(8010, 1544, 384, N.F16, N.F16, N.W_NK, 384, 384, 1544, 0, N.ACT_NONE, 512, 801, 1)
    assert lib.ancha_linear_workspace(C.byref(ld), C.byref(n)) == N.OK and n.value == 2 * 32 * 801 * 16
    ld0 = N.LinearDesc(8010, 1536, 384, N.F16, N.F16, N.W_NK, 384, 384, 1536, 0, N.ACT_GELU, 0, 1, 1)
    assert lib.ancha_linear_workspace(C.byref(ld0), C.byref(n)) == N.OK and n.value == 0
    assert lib.ancha_attention_workspace(None, C.byref(n)) == N.E_INVALID


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = N.lib()
    assert lib.ancha_attention_fwd(None, None, None, None, None, None, None) == N.E_INVALID
    d = N.AttnDesc(1, 1, 1, 32, N.F32, 64, 64, 1, 1, 0, 1, 0, 0, 0, -1, 0)
    # head_dim 32 is the reference's `None` (cuda_contracts.rs:249-250).
    assert lib.ancha_attention_fwd(C.byref(d), 1, 1, 1, None, 1, None) == N.E_UNSUPPORTED
    ld = N.LinearDesc(4, 128, 12, N.F32, N.F32, N.W_KN, 12, 128, 128, 0, N.ACT_NONE, 0, 1, 1)
    assert lib.ancha_linear_fwd(C.byref(ld), 1, 1, None, None, None, 1, None) != N.OK
    # A negative length is rejected before the status word behind the scratch is addressed
    # (without a GPU a device memset would answer with a CUDA error instead).
    for samples, hop in ((-100000, 1), (1024, 512), (44100, 2048)):
        assert lib.ancha_istft_masked(16, 16, 1, 1, samples, hop, 0, 16, 16, None) == N.E_INVALID
        assert "require hop" in N.last_error()
    assert lib.ancha_mdx_set_gemm(None, N.PRECISION_F16) == N.E_INVALID
    h = C.c_void_p()
    assert lib.ancha_model_load(b"/nonexistent-package", 0, 0, C.byref(h)) != N.OK
    assert not h.value


def test_model_load_rejects_an_invalid_manifest_before_device_work(tmp_path):
    """The manifest is read and validated before the device is touched, so without a GPU an
    invalid package still reports its own error (not a CUDA one)."""
    import json
    from ancha_b200 import synthetic
    pkg = tmp_path / "pkg"
    synthetic.tiny_package(str(pkg), "mel-band-roformer")
    m = json.loads((pkg / "manifest.json").read_text())
    m["config"]["hop"] = 2048
    (pkg / "manifest.json").write_text(json.dumps(m))
    h = C.c_void_p()
    assert N.lib().ancha_model_load(str(pkg).encode(), 0, N.PRECISION_F16, C.byref(h)) == N.E_INVALID
    assert "hop" in N.last_error() and not h.value
