"""Block blob format (pack + layout check) -- TEST INFRASTRUCTURE ONLY.

Restates the reference's on-disk unit so tests can feed the GPU library's
upload entry point exactly the bytes the reference's loader would map:

* packing: tools/pack_block.py:41-99 -- entries sorted by name, each offset
  rounded up to 64 bytes with zero fill, `name::q8` (int8 [O, I]) and
  `name::q8scale` (f32 [O, I/128]) companions beside a quantised weight,
  per-entry and whole-blob sha256.
* layout check: ltx/loader.zig:73-82 (aligned, gap < align, no trailing bytes).
* name normalisation: ltx/loader.zig:102-119 ('.' -> '_', '::' -> '_').

The golden test pins `pack()` byte-for-byte against the reference packer run
on the same fixture (tests/golden/make_golden.py).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np

from . import ltx_block_ref as ref

ALIGN = 64

# block field -> checkpoint tensor suffix (the dotted names whose
# normalised form is the file stem of ltx/block.zig:377-406)
DOTTED = {
    "q1_w": "attn1.to_q.weight", "q1_b": "attn1.to_q.bias",
    "k1_w": "attn1.to_k.weight", "k1_b": "attn1.to_k.bias",
    "v1_w": "attn1.to_v.weight", "v1_b": "attn1.to_v.bias",
    "o1_w": "attn1.to_out.0.weight", "o1_b": "attn1.to_out.0.bias",
    "qn1": "attn1.q_norm.weight", "kn1": "attn1.k_norm.weight",
    "g1_w": "attn1.to_gate_logits.weight", "g1_b": "attn1.to_gate_logits.bias",
    "q2_w": "attn2.to_q.weight", "q2_b": "attn2.to_q.bias",
    "k2_w": "attn2.to_k.weight", "k2_b": "attn2.to_k.bias",
    "v2_w": "attn2.to_v.weight", "v2_b": "attn2.to_v.bias",
    "o2_w": "attn2.to_out.0.weight", "o2_b": "attn2.to_out.0.bias",
    "qn2": "attn2.q_norm.weight", "kn2": "attn2.k_norm.weight",
    "g2_w": "attn2.to_gate_logits.weight", "g2_b": "attn2.to_gate_logits.bias",
    "ff1_w": "ff.net.0.proj.weight", "ff2_w": "ff.net.2.weight",
    "sst": "scale_shift_table", "psst": "prompt_scale_shift_table",
}


@dataclass
class Entry:
    name: str
    dtype: str          # "BF16" | "F32" | "I8"
    shape: list
    offset: int
    nbytes: int
    sha256: str


def normalize_name(name: str) -> str:
    """ltx/loader.zig:102-119."""
    return name.replace("::", "_").replace(".", "_")


def block_tensors(bw: ref.BlockWeights, block_idx: int = 0, scale_dtype_name: str | None = None):
    """(name, dtype, shape, bytes) for every stored tensor of one block, in
    the reference's naming (`transformer_blocks.{i}.<dotted>` + companions)."""
    out = []
    for field_, dotted in DOTTED.items():
        name = f"transformer_blocks.{block_idx}.{dotted}"
        a = bw.raw[field_]
        dt = "F32" if a.dtype == np.float32 else "BF16"
        out.append((name, dt, list(a.shape), a.tobytes()))
        if field_ + "::q8" in bw.raw:
            q = bw.raw[field_ + "::q8"]
            sc = bw.raw[field_ + "::q8scale"]
            out.append((name + "::q8", "I8", list(q.shape), q.tobytes()))
            sdt = "BF16" if sc.dtype == np.uint16 else "F32"
            out.append((name + "::q8scale", scale_dtype_name or sdt, list(sc.shape), sc.tobytes()))
    return out


def pack(tensors) -> tuple[bytes, list[Entry]]:
    """tools/pack_block.py:41-69 restated: name-sorted, 64-byte aligned."""
    blob = bytearray()
    entries = []
    for name, dt, shape, data in sorted(tensors, key=lambda t: t[0]):
        if len(blob) % ALIGN:
            blob.extend(b"\x00" * (ALIGN - len(blob) % ALIGN))
        off = len(blob)
        blob.extend(data)
        entries.append(Entry(name, dt, list(shape), off, len(data), hashlib.sha256(data).hexdigest()))
    return bytes(blob), entries


def check_layout(entries: list[Entry], total: int, align: int = ALIGN) -> None:
    """ltx/loader.zig:73-82; raises ValueError with the reference's error name."""
    end = 0
    for e in entries:
        if e.offset % align:
            raise ValueError("Misaligned")
        if e.offset < end or e.offset - end >= align:
            raise ValueError("LayoutGap")
        end = e.offset + e.nbytes
    if end != total:
        raise ValueError("TrailingBytes")


def block_weights_from_blob(data: bytes, entries, geom: ref.Geometry, block_idx: int = 0) -> ref.BlockWeights:
    """The inverse of block_tensors: one block's tensors read back from a
    packed blob (entries as dicts or Entry objects, names as the reference's
    loader finds them, ltx/loader.zig:102-129). A quantised field may be
    stored without its bf16 original (`name::q8` + `name::q8scale` only);
    its float tensor is then the exact f64 dequantisation."""
    import torch
    by_name = {}
    for e in entries:
        g = (lambda k: e[k]) if isinstance(e, dict) else (lambda k: getattr(e, k))
        by_name[normalize_name(g("name"))] = (g("dtype"), list(g("shape")), g("offset"), g("nbytes"))

    def read(key):
        dt, shape, off, nb = by_name[key]
        raw = np.frombuffer(data, dtype=np.uint8, count=nb, offset=off)
        npdt = {"BF16": np.uint16, "F32": np.float32, "I8": np.int8}[dt]
        return raw.view(npdt).reshape(shape).copy(), dt

    bw = ref.BlockWeights(geom=geom)
    for field_, dotted in DOTTED.items():
        key = normalize_name(f"transformer_blocks.{block_idx}.{dotted}")
        if key + "_q8" in by_name:
            q, _ = read(key + "_q8")
            sc, _ = read(key + "_q8scale")
            bw.raw[field_ + "::q8"] = q
            bw.raw[field_ + "::q8scale"] = sc
        if key in by_name:
            a, dt = read(key)
            bw.raw[field_] = a
            f = a if dt == "F32" else ref.bf16_to_f32(a)
            bw.t[field_] = torch.from_numpy(f.astype(np.float64))
        elif field_ + "::q8" in bw.raw:
            bw.t[field_] = torch.from_numpy(ref.dequant(bw.raw[field_ + "::q8"], bw.raw[field_ + "::q8scale"]))
        else:
            raise KeyError(f"blob has no entry {key}")
    return bw
