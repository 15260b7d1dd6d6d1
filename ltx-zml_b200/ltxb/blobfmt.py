"""The packed-blob format of the reference's weight units, as a writer.

A blob is every tensor of one unit (a transformer block, or the core parts)
sorted by name, each starting at a 64-byte-aligned offset with zero fill in
between, plus a manifest of (name, dtype, shape, offset, nbytes, sha256)
(tools/pack_block.py:41-99); int8 grouped-128 companions `<name>::q8` (int8
[O, I]) and `<name>::q8scale` ([O, I/128], f32 or bf16) sit beside the
quantised weights. `Blob.open` / `Blob.from_bytes` read it back and
`ltxb_weights_upload` / `ltxb_core_upload` take its entries.

BLOCK_TENSORS lists a block's tensors under their checkpoint names
(`transformer_blocks.<i>.<suffix>`, ltx/block.zig:377-406): bf16 except the
two f32 modulation tables.
"""

from __future__ import annotations

import hashlib
import json
import pathlib

ALIGN = 64

# (checkpoint suffix, shape in terms of D / H / FF, dtype)
BLOCK_TENSORS = [
    ("attn1.to_q.weight", ("D", "D"), "BF16"), ("attn1.to_q.bias", ("D",), "BF16"),
    ("attn1.to_k.weight", ("D", "D"), "BF16"), ("attn1.to_k.bias", ("D",), "BF16"),
    ("attn1.to_v.weight", ("D", "D"), "BF16"), ("attn1.to_v.bias", ("D",), "BF16"),
    ("attn1.to_out.0.weight", ("D", "D"), "BF16"), ("attn1.to_out.0.bias", ("D",), "BF16"),
    ("attn1.q_norm.weight", ("D",), "BF16"), ("attn1.k_norm.weight", ("D",), "BF16"),
    ("attn1.to_gate_logits.weight", ("H", "D"), "BF16"), ("attn1.to_gate_logits.bias", ("H",), "BF16"),
    ("attn2.to_q.weight", ("D", "D"), "BF16"), ("attn2.to_q.bias", ("D",), "BF16"),
    ("attn2.to_k.weight", ("D", "D"), "BF16"), ("attn2.to_k.bias", ("D",), "BF16"),
    ("attn2.to_v.weight", ("D", "D"), "BF16"), ("attn2.to_v.bias", ("D",), "BF16"),
    ("attn2.to_out.0.weight", ("D", "D"), "BF16"), ("attn2.to_out.0.bias", ("D",), "BF16"),
    ("attn2.q_norm.weight", ("D",), "BF16"), ("attn2.k_norm.weight", ("D",), "BF16"),
    ("attn2.to_gate_logits.weight", ("H", "D"), "BF16"), ("attn2.to_gate_logits.bias", ("H",), "BF16"),
    ("ff.net.0.proj.weight", ("FF", "D"), "BF16"),
    ("ff.net.2.weight", ("D", "FF"), "BF16"),
    ("scale_shift_table", (9, "D"), "F32"),
    ("prompt_scale_shift_table", (2, "D"), "F32"),
]

# the int8 set of the reference's quantised block (ltx/loader.zig:147-156) and
# its extension with the two output projections
Q8_REF = ("attn1.to_q.weight", "attn1.to_k.weight", "attn1.to_v.weight", "attn2.to_q.weight",
          "attn2.to_k.weight", "attn2.to_v.weight", "ff.net.0.proj.weight", "ff.net.2.weight")
Q8_EXT = Q8_REF + ("attn1.to_out.0.weight", "attn2.to_out.0.weight")


# the core parts' tensors (ltx/core_parts.zig:52-70), checkpoint names
CORE_TENSORS = [
    ("adaln_single.emb.timestep_embedder.linear_1.weight", ("D", 256), "BF16"),
    ("adaln_single.emb.timestep_embedder.linear_1.bias", ("D",), "BF16"),
    ("adaln_single.emb.timestep_embedder.linear_2.weight", ("D", "D"), "BF16"),
    ("adaln_single.emb.timestep_embedder.linear_2.bias", ("D",), "BF16"),
    ("adaln_single.linear.weight", ("9D", "D"), "BF16"),
    ("adaln_single.linear.bias", ("9D",), "BF16"),
    ("prompt_adaln_single.emb.timestep_embedder.linear_1.weight", ("D", 256), "BF16"),
    ("prompt_adaln_single.emb.timestep_embedder.linear_1.bias", ("D",), "BF16"),
    ("prompt_adaln_single.emb.timestep_embedder.linear_2.weight", ("D", "D"), "BF16"),
    ("prompt_adaln_single.emb.timestep_embedder.linear_2.bias", ("D",), "BF16"),
    ("prompt_adaln_single.linear.weight", ("2D", "D"), "BF16"),
    ("prompt_adaln_single.linear.bias", ("2D",), "BF16"),
    ("patchify_proj.weight", ("D", 128), "BF16"),
    ("patchify_proj.bias", ("D",), "BF16"),
    ("proj_out.weight", (128, "D"), "BF16"),
    ("proj_out.bias", (128,), "BF16"),
    ("scale_shift_table", (2, "D"), "F32"),
]


def shape_of(spec, d: int, ff: int = 0) -> list:
    m = {"D": d, "H": d // 128, "FF": ff, "9D": 9 * d, "2D": 2 * d}
    return [m.get(s, s) if isinstance(s, str) else s for s in spec]


def pack(tensors) -> tuple[bytes, list[dict]]:
    """tensors: (name, dtype "BF16" | "F32" | "I8", shape, bytes). Returns the
    blob bytes and the manifest entries (name-sorted, 64-byte aligned)."""
    blob = bytearray()
    entries = []
    for name, dt, shape, data in sorted(tensors, key=lambda t: t[0]):
        if len(blob) % ALIGN:
            blob.extend(b"\x00" * (ALIGN - len(blob) % ALIGN))
        off = len(blob)
        blob.extend(data)
        entries.append(dict(name=name, dtype=dt, shape=list(shape), offset=off, nbytes=len(data),
                            sha256=hashlib.sha256(data).hexdigest()))
    return bytes(blob), entries


def write_dir(directory, tensors, block: int = 0, provenance: dict | None = None) -> dict:
    """Writes the on-disk unit of tools/pack_block.py:41-99 into `directory`:
    blob.bin and blob_manifest.json (align, block, total_bytes, blob_sha256,
    entries with their own sha256, plus `provenance` fields such as repo and
    revision). Returns the manifest."""
    d = pathlib.Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    blob, entries = pack(tensors)
    man = dict(packer_version=1, packer_commit="ltxb", align=ALIGN, block=block, repo="", revision="",
               source_file="", model_version="")
    man.update(provenance or {})
    man.update(total_bytes=len(blob), blob_sha256=hashlib.sha256(blob).hexdigest(), entries=entries)
    (d / "blob.bin").write_bytes(blob)
    (d / "blob_manifest.json").write_text(json.dumps(man, indent=1))
    return man
