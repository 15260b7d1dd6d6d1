"""CPU tests of the C-ABI boundary: libltxb.so loads, exports exactly what
include/ltxb.h declares, and its host-only entry points (no GPU needed)
behave like the reference's loader checks (ltx/loader.zig:73-82)."""

import ctypes
import json
import pathlib
import re
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "ltxb.h"
GOLD = ROOT / "tests" / "golden" / "ref_tools"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ltxb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    fns = declared_functions()
    for must in ("ltxb_init", "ltxb_weights_upload", "ltxb_weights_free", "ltxb_block_forward",
                 "ltxb_attention", "ltxb_dq_gemm", "ltxb_last_error", "ltxb_comm_init"):
        assert must in fns


def test_library_exports_every_declared_symbol():
    import ltxb
    out = subprocess.run(["nm", "-D", "--defined-only", str(ltxb.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s(ltxb_[a-z0-9_]+)$", out, flags=re.M))
    missing = [f for f in declared_functions() if f not in exported]
    assert not missing, f"declared in ltxb.h but not exported: {missing}"
    for f in declared_functions():
        assert hasattr(ltxb.lib, f)


def test_version_and_error_string():
    import ltxb
    assert "sm_100a" in ltxb.version()
    assert isinstance(ltxb.last_error(), str)


def _golden_blob():
    import ltxb
    return ltxb.Blob.open(GOLD, verify_digest=True)


def test_blob_open_and_layout_ok():
    b = _golden_blob()
    b.check_layout()
    e = b.find_entry("transformer_blocks_0_attn1_to_q_weight_q8scale")
    assert e["dtype"] == "F32" and e["shape"] == [32, 2]


@pytest.mark.parametrize("mutate,err", [
    (lambda es: es[1].__setitem__("offset", es[1]["offset"] + 4), "Misaligned"),
    (lambda es: es[1].__setitem__("offset", es[1]["offset"] + 64), "LayoutGap"),
    (lambda es: es.pop(), "TrailingBytes"),
])
def test_blob_layout_errors(mutate, err):
    import ltxb
    man = json.loads((GOLD / "blob_manifest.json").read_text())
    entries = [dict(e) for e in man["entries"]]
    mutate(entries)
    b = ltxb.Blob(b"", {"align": 64, "total_bytes": man["total_bytes"], "entries": entries})
    with pytest.raises(ltxb.LtxbError) as ei:
        b.check_layout()
    assert ei.value.code == ltxb.ELAYOUT and err in str(ei.value)


def test_missing_entry_error():
    import ltxb
    with pytest.raises(ltxb.LtxbError) as ei:
        _golden_blob().find_entry("transformer_blocks_0_nope")
    assert ei.value.code == ltxb.EMISSING


def test_blob_size_mismatch(tmp_path):
    import ltxb
    (tmp_path / "blob.bin").write_bytes((GOLD / "blob.bin").read_bytes()[:-1])
    (tmp_path / "blob_manifest.json").write_text((GOLD / "blob_manifest.json").read_text())
    with pytest.raises(ltxb.LtxbError, match="BlobSizeMismatch"):
        ltxb.Blob.open(tmp_path)


def test_blob_digest_mismatch(tmp_path):
    import ltxb
    data = bytearray((GOLD / "blob.bin").read_bytes())
    data[100] ^= 1
    (tmp_path / "blob.bin").write_bytes(bytes(data))
    (tmp_path / "blob_manifest.json").write_text((GOLD / "blob_manifest.json").read_text())
    with pytest.raises(ltxb.LtxbError, match="BlobDigestMismatch"):
        ltxb.Blob.open(tmp_path, verify_digest=True)


def test_null_arguments_rejected():
    import ltxb
    assert ltxb.lib.ltxb_blob_check_layout(None, 3, 0, 64) == ltxb.EINVAL
    h = ctypes.c_void_p()
    assert ltxb.lib.ltxb_weights_upload(0, None, 0, None, 0, 0, 0, 0, 4096, 16384, ctypes.byref(h)) == ltxb.EINVAL
    ltxb.lib.ltxb_weights_free(None)
    ltxb.lib.ltxb_comm_free(None)


def test_blob_writer_matches_reference_packer():
    """The library's blob writer (ltxb.blobfmt) produces byte-for-byte the
    format the oracle restates from tools/pack_block.py."""
    import numpy as np
    from ltxb import blobfmt
    from oracle import blob as oblob
    from oracle import inputs as oin
    from oracle import ltx_block_ref as ref
    geom = ref.Geometry(d=256, ff=512)
    bw = oin.make_weights(geom, 3, quant="int8")
    tensors = oblob.block_tensors(bw, 2)
    data_o, ent_o = oblob.pack(tensors)
    data_l, ent_l = blobfmt.pack(tensors)
    assert data_o == data_l
    assert [(e.name, e.offset, e.nbytes, e.sha256) for e in ent_o] == \
        [(e["name"], e["offset"], e["nbytes"], e["sha256"]) for e in ent_l]
    names = {e.name[len("transformer_blocks.2."):] for e in ent_o if "::" not in e.name}
    assert names == {suffix for suffix, _, _ in blobfmt.BLOCK_TENSORS}
    assert set(blobfmt.Q8_REF) == {oblob.DOTTED[f] for f in ref.Q8_FIELDS}
    assert set(blobfmt.Q8_EXT) == {oblob.DOTTED[f] for f in ref.Q8_FIELDS_EXT}
    for suffix, spec, dt in blobfmt.BLOCK_TENSORS:
        e = next(x for x in ent_o if x.name == "transformer_blocks.2." + suffix)
        assert list(e.shape) == blobfmt.shape_of(spec, 256, 512) and e.dtype == dt


def test_core_tensor_list_matches_oracle():
    from ltxb import blobfmt
    from oracle import core_ref as cr
    got = [(n, blobfmt.shape_of(sp, 512), dt) for n, sp, dt in blobfmt.CORE_TENSORS]
    want = [(n, list(shape(512)), "F32" if dt == "f32" else "BF16") for n, shape, dt in cr.CORE_SPECS.values()]
    assert sorted(got) == sorted(want)


# Fake device addresses: the operator entry points must reject these
# arguments on the host, before any CUDA call (none of them is dereferenced).
_A, _W, _O, _WS, _SC = 0x10000, 0x20000, 0x30000, 0x40000, 0x50000


@pytest.mark.parametrize("call,msg", [
    (lambda l, p: l.ltxb_gemm_bf16(p(_A), p(_W), None, p(_O + 8), 128, 256, 64, None), "16-byte aligned"),
    (lambda l, p: l.ltxb_gemm_bf16(p(_A), p(_W), p(_SC + 2), p(_O), 128, 256, 64, None), "16-byte aligned"),
    (lambda l, p: l.ltxb_gemm_bf16(p(_A + 4), p(_W), None, p(_O), 128, 256, 64, None), "16-byte aligned"),
    (lambda l, p: l.ltxb_gemm_bf16(p(_A), p(_W), None, p(_O), 128, 256, 96, None), "multiple of 64"),
    (lambda l, p: l.ltxb_gemm_bf16(p(_A), p(_W), None, p(_O), 128, 48, 64, None), "multiple of 32"),
    (lambda l, p: l.ltxb_gemm_bf16(p(_A), p(_W), None, p(_O), 0, 256, 64, None), "empty shape"),
    (lambda l, p: l.ltxb_dq_gemm(p(_A), p(_W + 1), p(_SC), 1, None, p(_O), 128, 256, 128, 0, p(_WS), 1 << 20,
                                 None), "16-byte aligned"),
    (lambda l, p: l.ltxb_dq_gemm(p(_A), p(_W), p(_SC + 2), 1, None, p(_O), 128, 256, 128, 0, p(_WS), 1 << 20,
                                 None), "element-aligned"),
    (lambda l, p: l.ltxb_dq_gemm(p(_A), p(_W), p(_SC), 1, None, p(_O), 128, 256, 128, 0, p(_WS), 1024, None),
     "workspace"),
    (lambda l, p: l.ltxb_dq_gemm(p(_A), p(_W), p(_SC), 1, None, p(_O), 128, 256, 64, 1, None, 0, None), "K % 128"),
    (lambda l, p: l.ltxb_dq_gemm(p(_A), p(_W), p(_SC), 7, None, p(_O), 128, 256, 128, 1, None, 0, None),
     "scale dtype"),
    (lambda l, p: l.ltxb_attention(p(_A + 2), p(_W), p(_SC), p(_O), None, 128, 128, 2, ctypes.c_float(0.1), None),
     "16-byte aligned"),
    (lambda l, p: l.ltxb_attention(p(_A), p(_W), p(_SC), p(_O), None, 128, 0, 2, ctypes.c_float(0.1), None),
     "empty K/V"),
    (lambda l, p: l.ltxb_attention_split(p(_A), p(_W), p(_SC), p(_O), None, 128, 512, 2, ctypes.c_float(0.1), -1,
                                         p(_WS), 1 << 30, None), "negative split"),
    (lambda l, p: l.ltxb_attention_split(p(_A), p(_W), p(_SC), p(_O), None, 128, 512, 2, ctypes.c_float(0.1), 2,
                                         p(_WS), 4096, None), "workspace"),
    (lambda l, p: l.ltxb_attention_split(p(_A), p(_W), p(_SC), p(_O), None, 128, 512, 2, ctypes.c_float(0.1), 2,
                                         p(_WS + 16), 1 << 30, None), "256-byte aligned"),
])
def test_operator_arguments_rejected_on_the_host(call, msg):
    """Misaligned operands and unsupported shapes return LTXB_EINVAL with a
    message before anything reaches the device (a misaligned 16-byte vector
    access or TMA copy would otherwise fault the GPU)."""
    import ltxb
    rc = call(ltxb.lib, ctypes.c_void_p)
    assert rc == ltxb.EINVAL, (rc, ltxb.last_error())
    assert msg in ltxb.last_error()
