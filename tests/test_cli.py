"""The sml-gpu-fwd command line (sheep_b200/cli/sml_gpu_fwd.c): it is built
beside the library and answers its usage line without touching a GPU."""
import os
import subprocess

from sheep_b200 import build


def test_cli_usage_without_a_gpu():
    exe = build.build_cli()
    assert os.access(exe, os.X_OK)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2
    assert r.stdout.startswith("usage: sml-gpu-fwd MODEL.ssf ids,comma,separated NGEN")
