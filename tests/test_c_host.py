"""The C ABI from plain C (no Python, no torch): tests/c_host/abi_host.c is
compiled with gcc against include/ltxb.h, linked to libltxb.so, and run. It
covers the host-side entry points a Zig or C caller uses before any GPU
work (blob layout check, ring schedule, sigma lists, error reporting)."""

import pathlib
import shutil
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
LIB_DIR = ROOT / "ltx-zml_b200" / "ltxb"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_host_program(tmp_path):
    if not (LIB_DIR / "libltxb.so").exists():
        pytest.skip("libltxb.so not built")
    exe = tmp_path / "abi_host"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_host" / "abi_host.c"), "-L", str(LIB_DIR), "-lltxb",
                    "-Wl,-rpath," + str(LIB_DIR), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout
