"""Mutation fuzzing of the classic MDX ONNX reader, graph builder and shape inference under
AddressSanitizer / UBSan (tests/fuzz_onnx_reader.cpp compiled with onnx.cpp). A model file is
untrusted input: no mutation may read out of bounds, overflow, or yield shapes whose kernel
indices leave 32 bits."""
import pathlib
import shutil
import subprocess
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_onnx_reader_survives_mutations(tmp_path):
    sys.path.insert(0, str(ROOT / "tests"))
    import test_gpu_mdx as G  # graph builders only; nothing here touches a GPU
    import test_oracle_mdx as T
    seeds = [T.fold_graph(), T.chain_graph(), G.tfc_tdf_graph(f=16, t=8)[0], G.shape_preserving_graph()]
    paths = []
    for i, b in enumerate(seeds):
        paths.append(tmp_path / f"seed{i}.onnx")
        paths[-1].write_bytes(b)
    exe = tmp_path / "fuzz"
    csrc = ROOT / "ancha_b200" / "csrc"
    build = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined",
                            "-fno-sanitize-recover=undefined", f"-I{csrc}", str(ROOT / "tests" / "fuzz_onnx_reader.cpp"),
                            str(csrc / "onnx.cpp"), "-o", str(exe)], capture_output=True, text=True, timeout=300)
    if build.returncode != 0 and "sanitize" in build.stderr:
        pytest.skip("sanitizer runtime unavailable: " + build.stderr.strip().splitlines()[-1])
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe), "20000", "7"] + [str(p) for p in paths], capture_output=True, text=True,
                         timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr[-4000:]
    assert "ERROR" not in run.stderr and "runtime error" not in run.stderr, run.stderr[-4000:]
    counts = dict(zip(run.stdout.split()[0::2], map(int, run.stdout.split()[1::2])))
    assert counts["accepted"] > 0 and counts["inferred"] > 0 and counts["convs"] > 0, run.stdout
