"""Mutation fuzzing of the host-side file formats (manifest JSON, safetensors, WAV) under
AddressSanitizer / UBSan: tests/fuzz_host_formats.cpp compiled with ancha_b200/csrc/hostio.cpp.
A model package and an input track are untrusted files; directed cases cover deep nesting,
integers a double cannot hold, bad escapes, tensor offsets whose sum wraps and element counts
whose byte size wraps."""
import pathlib
import shutil
import struct
import subprocess

import numpy as np
import pytest

from ancha_b200 import synthetic as S

ROOT = pathlib.Path(__file__).resolve().parents[1]


def _wav(path):
    pcm = (np.random.default_rng(0).standard_normal((200, 2)) * 3000).astype("<i2").tobytes()
    fmt = struct.pack("<HHIIHH", 1, 2, 44100, 44100 * 4, 4, 16)
    body = (b"WAVEfmt " + struct.pack("<I", 16) + fmt + b"LIST" + struct.pack("<I", 3) + b"abc\0" + b"data"
            + struct.pack("<I", len(pcm)) + pcm)
    path.write_bytes(b"RIFF" + struct.pack("<I", len(body)) + body)


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_host_formats_survive_mutations(tmp_path):
    S.tiny_package(str(tmp_path / "pkg"), "mel-band-roformer")
    S.write_safetensors(str(tmp_path / "small.safetensors"),
                        {"a.weight": np.ones((3, 4), np.float32), "b": np.arange(5, dtype=np.float32),
                         "c.gamma": np.zeros((2, 1, 2), np.float32)})
    _wav(tmp_path / "track.wav")
    exe = tmp_path / "fuzz"
    csrc = ROOT / "ancha_b200" / "csrc"
    build = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined",
                            "-fno-sanitize-recover=undefined", f"-I{csrc}", str(ROOT / "tests" / "fuzz_host_formats.cpp"),
                            str(csrc / "hostio.cpp"), "-o", str(exe)], capture_output=True, text=True, timeout=300)
    if build.returncode != 0 and "sanitize" in build.stderr:
        pytest.skip("sanitizer runtime unavailable: " + build.stderr.strip().splitlines()[-1])
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe), "3000", "11", str(tmp_path / "scratch.wav"), str(tmp_path / "pkg" / "manifest.json"),
                          str(tmp_path / "small.safetensors"), str(tmp_path / "track.wav")],
                         capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr[-4000:]
    assert "ERROR" not in run.stderr and "runtime error" not in run.stderr, run.stderr[-4000:]
    f = run.stdout.split()
    counts = {f[i]: (int(f[i + 1]), int(f[i + 2])) for i in range(0, len(f), 3)}
    assert all(ok > 0 and bad > 0 for ok, bad in counts.values()), run.stdout  # both outcomes exercised
