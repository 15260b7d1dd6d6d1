#!/usr/bin/env python3
"""Regenerate the golden fixtures under tests/golden/ref_tools/ by running the
reference's OWN Python tools on a small synthetic block.

    python tests/golden/make_golden.py /path/to/reference

This needs the reference checkout (its `tools/` directory) and runs only in
the build container; the committed outputs travel with the repo, so tests on
the GPU box read the fixtures and never the reference.

What it pins:
* tools/quantize_block.py (int8, grouped-128, the qkv and ff classes exactly
  as tools/assemble_blocks.py:80-81 invokes it) -> *_q8.bin / *_q8scale.bin
* tools/pack_block.py -> blob.bin + blob_manifest.json

The synthetic block is a scaled-down LTX block dir in fetch_block.py's
manifest format (tools/fetch_block.py:152-178): bf16 tensors with the real
names, N(0, 0.02) weights, 0.5% outlier input channels x20, one all-zero
weight row and one all-zero group (absmax == 0 -> scale 1.0).
"""

import hashlib
import json
import pathlib
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "ref_tools"

# (dotted name, shape, dtype) of the fixture block
TENSORS = [
    ("attn1.to_q.weight", (32, 256), "BF16"),
    ("attn1.to_q.bias", (32,), "BF16"),
    ("attn1.to_k.weight", (32, 256), "BF16"),
    ("attn1.to_v.weight", (32, 256), "BF16"),
    ("attn1.to_out.0.weight", (32, 32), "BF16"),
    ("ff.net.0.proj.weight", (64, 256), "BF16"),
    ("ff.net.2.weight", (32, 384), "BF16"),
    ("scale_shift_table", (9, 32), "F32"),
]
BLOCK = 0


def bf16_bits(a):
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def make_tensor(name, shape, dtype, rng):
    a = (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if len(shape) == 2 and name.endswith("weight"):
        k = shape[1]
        cols = rng.choice(k, size=max(1, round(0.005 * k)), replace=False)
        a[:, cols] *= np.float32(20.0)
        a[3, :] = 0.0                                   # absmax == 0 row
        a[5, :128] = 0.0                                # one all-zero group
    if dtype == "BF16":
        return bf16_bits(a).tobytes()
    return a.astype(np.float32).tobytes()


def main() -> int:
    if len(sys.argv) < 2:
        print("usage: make_golden.py <checkout of the reference repository>", file=sys.stderr)
        return 2
    ref_root = pathlib.Path(sys.argv[1])
    tools = ref_root / "tools"
    rng = np.random.default_rng(20260821)
    with tempfile.TemporaryDirectory() as td:
        wdir = pathlib.Path(td) / "block"
        wdir.mkdir()
        man = {"repo": "synthetic/fixture", "revision": "0" * 40, "file": "fixture.safetensors",
               "block": BLOCK, "header_sha256": "0" * 64, "model_version": "fixture", "tensors": {}}
        for dotted, shape, dtype in TENSORS:
            short = f"transformer_blocks.{BLOCK}.{dotted}"
            data = make_tensor(dotted, shape, dtype, rng)
            fname = short.replace(".", "_") + ".bin"
            (wdir / fname).write_bytes(data)
            man["tensors"][short] = {"file": fname, "shape": list(shape), "dtype": dtype,
                                     "sha256": hashlib.sha256(data).hexdigest()}
        (wdir / "manifest.json").write_text(json.dumps(man, indent=1))
        for cls in ("qkv", "ff"):
            subprocess.run([sys.executable, str(tools / "quantize_block.py"), str(wdir),
                            "--cls", cls, "--gs", "128", "--bits", "8"], check=True)
        subprocess.run([sys.executable, str(tools / "pack_block.py"), str(wdir)], check=True)
        if OUT.exists():
            shutil.rmtree(OUT)
        OUT.mkdir(parents=True)
        for p in sorted(wdir.iterdir()):
            shutil.copy(p, OUT / p.name)
    # the packer records the tools checkout's git commit; pin it to a constant
    bm = json.loads((OUT / "blob_manifest.json").read_text())
    bm["packer_commit"] = "fixture"
    (OUT / "blob_manifest.json").write_text(json.dumps(bm, indent=1))
    print(f"wrote {len(list(OUT.iterdir()))} files to {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
