"""The C ABI from plain C (no Python, no torch): tests/c_host/abi_host.c is
compiled with gcc against include/ltxb.h, linked to libltxb.so, and run. It
covers the host-side entry points a Zig or C caller uses before any GPU
work (blob layout check, the native blob reader on the reference packer's
output, ring schedule, sigma lists, error reporting)."""

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
    r = subprocess.run([str(exe), str(ROOT / "tests" / "golden" / "ref_tools")], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout and "ok blob: open with both digest checks" in r.stdout


@pytest.mark.gpu
@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_host_runs_a_block(cuda, tmp_path):
    """tests/c_host/block_host.c -- a C program using only include/ltxb.h and
    the CUDA driver API for its own buffers -- uploads an int8 block from a
    packed blob and runs ltxb_block_forward; its output equals the Python
    mirror's call of the same entry point bit for bit and the oracle within
    the block's 5e-3."""
    import numpy as np
    import torch

    import helpers
    import ltxb
    from oracle import ltx_block_ref as ref

    cuda_root = pathlib.Path("/usr/local/cuda")
    stubs = cuda_root / "lib64" / "stubs"
    if not (cuda_root / "include" / "cuda.h").exists() or not (stubs / "libcuda.so").exists():
        pytest.skip("CUDA driver headers / link stub not found")
    d, ff, grid, s = 256, 512, (2, 4, 8), 16
    geom, bw, data, ent, qset = helpers.weights_case(d, ff, 4, "int8")
    inp = helpers.inputs_case(d, grid, s, 4, "axes", 3, "random")
    T, K = inp.x.shape[0], inp.tstab.shape[0]
    dt = {"BF16": 0, "F32": 1, "I8": 2}
    (tmp_path / "blob.bin").write_bytes(data)
    with open(tmp_path / "manifest.txt", "w") as f:
        for e in ent:
            shape = list(e["shape"]) + [0] * (2 - len(e["shape"]))
            f.write(f"{e['name']} {dt[e['dtype']]} {len(e['shape'])} {shape[0]} {shape[1]} {e['offset']} "
                    f"{e['nbytes']}\n")
    (tmp_path / "dims.txt").write_text(f"{T} {s} {K} {d} {ff} {ltxb.MODE_INT8} {ltxb.QSET_REF}\n")
    with open(tmp_path / "inputs.bin", "wb") as f:
        for a, t in ((inp.x, np.float32), (inp.tstab, np.float32), (inp.tidx, np.int32), (inp.ctx, np.float32),
                     (inp.pts2, np.float32), (inp.cos, np.float32), (inp.sin, np.float32)):
            f.write(np.ascontiguousarray(a, dtype=t).tobytes())
    exe = tmp_path / "block_host"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-I",
                    str(cuda_root / "include"), str(ROOT / "tests" / "c_host" / "block_host.c"), "-L",
                    str(LIB_DIR), "-lltxb", "-Wl,-rpath," + str(LIB_DIR), "-L", str(stubs), "-lcuda", "-o",
                    str(exe)], check=True)
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    got = np.fromfile(tmp_path / "out.bin", dtype=np.float32).reshape(T, d)
    w = helpers.upload(data, ent, geom, ltxb.MODE_INT8)
    mine = ltxb.QBlock(w).forward(*helpers.to_cuda(inp, cuda))
    torch.cuda.synchronize()
    assert np.array_equal(got, mine.cpu().numpy())
    want = helpers.oracle_stages(bw, inp, qset)["block_out"]
    assert ref.rel_rms(got, want) < 5e-3
    w.free()


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
@pytest.mark.parametrize("sanitizer", ["address,undefined", "thread"])
def test_host_code_under_sanitizers(tmp_path, sanitizer):
    """The library's host-only C++ -- the blob reader and the staging ring --
    built with tests/c_host/host_sanitize.cpp under AddressSanitizer + UBSan
    (3,000 mutated manifests through ltxb_blob_open) and under
    ThreadSanitizer (the staging ring's reader thread against the consumer,
    with early ends, aborts and teardown). Any report fails the test."""
    import os

    import numpy as np

    from ltxb import blobfmt
    cuda = pathlib.Path("/usr/local/cuda")
    if not (cuda / "include" / "cuda_runtime.h").exists():
        pytest.skip("CUDA headers not found")
    csrc = ROOT / "ltx-zml_b200" / "csrc"
    exe = tmp_path / "host_sanitize"
    subprocess.run(["g++", "-std=c++17", "-O1", "-g", f"-fsanitize={sanitizer}", "-fno-sanitize-recover=all",
                    "-I", str(ROOT / "include"), "-I", str(cuda / "include"),
                    str(ROOT / "tests" / "c_host" / "host_sanitize.cpp"), str(csrc / "blob.cpp"),
                    str(csrc / "stage.cpp"), "-L", str(cuda / "lib64"), "-lcudart",
                    "-Wl,-rpath," + str(cuda / "lib64"), "-lpthread", "-o", str(exe)], check=True)
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", TSAN_OPTIONS="halt_on_error=1")
    if sanitizer.startswith("address"):
        work = tmp_path / "work"
        work.mkdir()
        args = ["fuzz", str(ROOT / "tests" / "golden" / "ref_tools"), str(work), "3000"]
    else:
        rng = np.random.default_rng(0)
        args = ["stage"]
        for i, n in enumerate([40000, 120000, 8000]):
            tensors = [(f"transformer_blocks.{i}.t{j}", "F32", [n // 4],
                        rng.standard_normal(n // 4).astype(np.float32).tobytes()) for j in range(3)]
            blobfmt.write_dir(tmp_path / f"b{i}", tensors, block=i)
            args.append(str(tmp_path / f"b{i}"))
    r = subprocess.run([str(exe)] + args, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]
    assert "Sanitizer" not in r.stderr, r.stderr[-4000:]
