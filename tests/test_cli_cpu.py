"""The separate command line (ancha_b200/cli.py): the reference's flags map onto
SeparateOptions, usage errors exit 2, and an engine error exits 1 with its message (no GPU
here, so the engine reports one)."""
import subprocess
import sys

import pytest

from ancha_b200 import cli
from ancha_b200.model import SeparateOptions


def parse(*argv):
    return cli.options(cli.parser().parse_args(["separate", *argv]))


def test_reference_flags_map_onto_separate_options():
    o = parse("song.wav", "--model", "pkg", "-o", "out", "--backend", "cuda", "--device", "3", "--start", "1.5",
              "--duration", "30", "--chunk-samples", "352800", "--overlap", "2", "--precision", "f16",
              "--batch-chunks", "4")
    assert o == SeparateOptions(input="song.wav", model="pkg", output="out", chunk_samples=352800, overlap=2,
                                precision="f16", batch_chunks=4, start_seconds=1.5, duration_seconds=30.0,
                                devices=[3])
    assert parse("a.wav", "--model", "p", "--output", "o", "--devices", "0,1,2").devices == [0, 1, 2]
    d = parse("a.wav", "--model", "p", "-o", "o")
    assert (d.devices, d.precision, d.chunk_samples, d.overlap) == ([0], "f16", None, None)


@pytest.mark.parametrize("argv", [["--backend", "cpu"], ["--device", "0", "--devices", "1"], ["--devices", "x"],
                                  ["--duration", "0"], ["--start", "-1"]])
def test_usage_errors(argv, capsys):
    assert cli.main(["separate", "a.wav", "--model", "p", "-o", "o", *argv]) == 2
    assert "error:" in capsys.readouterr().err


def test_engine_error_exits_1_with_its_message(tmp_path):
    r = subprocess.run([sys.executable, "-m", "ancha_b200", "separate", str(tmp_path / "missing.wav"), "--model",
                        str(tmp_path / "pkg"), "-o", str(tmp_path / "out")], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 1 and "error:" in r.stderr and not (tmp_path / "out").exists()
