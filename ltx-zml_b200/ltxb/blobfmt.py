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
    blob, entries = pack(tensors)
    return write_packed(directory, blob, entries, block, provenance)


def write_packed(directory, blob: bytes, entries: list, block: int = 0, provenance: dict | None = None) -> dict:
    """write_dir for a blob already packed (e.g. by synthetic_block)."""
    d = pathlib.Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    man = dict(packer_version=1, packer_commit="ltxb", align=ALIGN, block=block, repo="", revision="",
               source_file="", model_version="")
    man.update(provenance or {})
    man.update(total_bytes=len(blob), blob_sha256=hashlib.sha256(blob).hexdigest(), entries=entries)
    (d / "blob.bin").write_bytes(blob)
    (d / "blob_manifest.json").write_text(json.dumps(man, indent=1))
    return man


def synthetic_block(device, d: int = 4096, ff: int = 16384, seed: int = 0, block: int = 0, q8=Q8_EXT,
                    outlier_frac: float = 0.005, outlier_mult: float = 20.0):
    """A seeded synthetic block in this format:
    weights N(0, 0.02) drawn on `device` (norm weights 1 + N(0, 0.02), the
    two modulation tables f32); every weight in `q8` gets 0.5% of its input
    channels scaled x20, then symmetric int8 grouped-128 quantisation with
    scale = absmax / 127 rounded to bf16 (q from the rounded scale), stored
    as `::q8` / `::q8scale` only. Returns (blob bytes, entries)."""
    import torch
    g = torch.Generator(device=device)
    tensors = []
    for i, (suffix, spec, dt) in enumerate(BLOCK_TENSORS):
        shape = shape_of(spec, d, ff)
        g.manual_seed(seed * 1000 + i)
        w = torch.randn(*shape, generator=g, device=device) * 0.02
        name = f"transformer_blocks.{block}.{suffix}"
        if dt == "F32":
            tensors.append((name, "F32", shape, w.cpu().numpy().tobytes()))
            continue
        if "norm" in suffix:
            w = w + 1.0
        if suffix in q8:
            k = shape[1]
            cols = torch.randperm(k, generator=g, device=device)[: max(1, round(outlier_frac * k))]
            w[:, cols] *= outlier_mult
            wg = w.view(shape[0], k // 128, 128)
            amax = wg.abs().amax(-1, keepdim=True)
            sc = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax)).to(torch.bfloat16)
            q = torch.clamp(torch.round(wg / sc.float()), -128, 127).to(torch.int8).view(shape)
            tensors.append((name + "::q8", "I8", shape, q.cpu().numpy().tobytes()))
            tensors.append((name + "::q8scale", "BF16", [shape[0], k // 128],
                            sc.view(torch.int16).view(shape[0], k // 128).cpu().numpy().tobytes()))
        else:
            tensors.append((name, "BF16", shape, w.to(torch.bfloat16).view(torch.int16).cpu().numpy().tobytes()))
    return pack(tensors)
