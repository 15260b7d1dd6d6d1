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
    ltxb.lib.ltxb_comm_abort(None)
    assert ltxb.lib.ltxb_comm_peer_mapped(None) == 0  # no communicator: no peer windows


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


# ---- the native blob reader (ltxb_blob_*) and its SHA-256 ----

def _sha_hex(lib, data: bytes) -> str:
    out = ctypes.create_string_buffer(65)
    buf = ctypes.create_string_buffer(data, len(data)) if data else None
    lib.ltxb_sha256_hex(buf, len(data), out)
    return out.value.decode()


@pytest.mark.parametrize("portable", [1, 0])
def test_sha256_matches_hashlib(portable):
    """FIPS 180-4 SHA-256 of the library against hashlib: every length 0..300
    (all padding cases) and a few large buffers, for the portable code and
    (where the CPU has them) the x86 SHA extensions."""
    import hashlib
    import os

    import ltxb
    lib = ltxb.lib
    try:
        lib.ltxb_sha256_impl(portable)
        for n in list(range(0, 301)) + [4096, 65537, 1 << 20]:
            data = os.urandom(n)
            assert _sha_hex(lib, data) == hashlib.sha256(data).hexdigest(), n
    finally:
        lib.ltxb_sha256_impl(0)


def _view(lib, h):
    p, nb, ent, n = ctypes.c_void_p(), ctypes.c_uint64(), ctypes.c_void_p(), ctypes.c_int()
    al, blk = ctypes.c_uint32(), ctypes.c_int64()
    assert lib.ltxb_blob_view(h, ctypes.byref(p), ctypes.byref(nb), ctypes.byref(ent), ctypes.byref(n),
                              ctypes.byref(al), ctypes.byref(blk)) == 0
    import ltxb
    arr = (ltxb._Entry * n.value).from_address(ent.value) if n.value else []
    return p.value, nb.value, list(arr), al.value, blk.value


def test_native_blob_open_matches_manifest():
    """ltxb_blob_open on the reference packer's output: both digest checks
    pass, the mapped bytes are blob.bin, every entry equals the manifest's
    (name, dtype, shape, offset, nbytes), and findEntry works."""
    import ltxb
    lib = ltxb.lib
    h = ctypes.c_void_p()
    assert lib.ltxb_blob_open(str(GOLD).encode(), ltxb.VERIFY_BLOB | ltxb.VERIFY_ENTRIES, ctypes.byref(h)) == 0, \
        ltxb.last_error()
    try:
        p, nb, ents, al, blk = _view(lib, h)
        raw = (GOLD / "blob.bin").read_bytes()
        assert nb == len(raw) and ctypes.string_at(p, nb) == raw
        man = json.loads((GOLD / "blob_manifest.json").read_text())
        assert al == man["align"] and blk == man["block"] and len(ents) == len(man["entries"])
        for e, m in zip(ents, man["entries"]):
            assert e.name.decode() == m["name"]
            assert e.dtype == {"BF16": 0, "F32": 1, "I8": 2}[m["dtype"]]
            assert e.ndim == len(m["shape"]) and list(e.shape)[:e.ndim] == m["shape"]
            assert (e.offset, e.nbytes) == (m["offset"], m["nbytes"])
        out = ctypes.c_void_p()
        assert lib.ltxb_blob_find(h, b"transformer_blocks_0_attn1_to_q_weight_q8scale", ctypes.byref(out)) == 0
        found = ltxb._Entry.from_address(out.value)
        assert found.name.decode() == "transformer_blocks.0.attn1.to_q.weight::q8scale" and found.dtype == 1
        assert lib.ltxb_blob_find(h, b"transformer_blocks_0_nope", ctypes.byref(out)) == ltxb.EMISSING
        assert lib.ltxb_blob_verify(h, ltxb.VERIFY_BLOB | ltxb.VERIFY_ENTRIES) == 0
    finally:
        lib.ltxb_blob_close(h)


def _blob_dir(tmp_path, data: bytes, manifest_text: str):
    (tmp_path / "blob.bin").write_bytes(data)
    (tmp_path / "blob_manifest.json").write_text(manifest_text)
    return str(tmp_path).encode()


def _open_rc(d, flags=0):
    import ltxb
    h = ctypes.c_void_p()
    rc = ltxb.lib.ltxb_blob_open(d, flags, ctypes.byref(h))
    if rc == 0:
        ltxb.lib.ltxb_blob_close(h)
    return rc, ltxb.last_error()


def test_native_blob_errors(tmp_path):
    """The loader's error cases through the native reader: missing files,
    size and digest mismatches (whole blob and one entry), layout errors and
    malformed manifests."""
    import ltxb
    raw = (GOLD / "blob.bin").read_bytes()
    mtext = (GOLD / "blob_manifest.json").read_text()
    man = json.loads(mtext)
    assert _open_rc(str(tmp_path / "none").encode())[0] == ltxb.EMISSING
    rc, msg = _open_rc(_blob_dir(tmp_path, raw[:-1], mtext))
    assert rc == ltxb.ELAYOUT and "BlobSizeMismatch" in msg
    bad = bytearray(raw)
    e3 = man["entries"][3]
    bad[e3["offset"] + 5] ^= 0x40
    d = _blob_dir(tmp_path, bytes(bad), mtext)
    assert _open_rc(d)[0] == 0  # no digest asked for
    rc, msg = _open_rc(d, ltxb.VERIFY_BLOB)
    assert rc == ltxb.ELAYOUT and "BlobDigestMismatch" in msg
    rc, msg = _open_rc(d, ltxb.VERIFY_ENTRIES)
    assert rc == ltxb.ELAYOUT and "BlobDigestMismatch" in msg and e3["name"] in msg
    m2 = json.loads(mtext)
    m2["entries"][1]["offset"] += 4
    rc, msg = _open_rc(_blob_dir(tmp_path, raw, json.dumps(m2)))
    assert rc == ltxb.ELAYOUT and "Misaligned" in msg
    for text, what in [(mtext[:-20], "truncated"), ("[]", "not an object"),
                       (json.dumps({k: v for k, v in man.items() if k != "total_bytes"}), "total_bytes"),
                       (json.dumps(dict(man, entries={})), "entries"),
                       ("[" * 100 + "]" * 100, "nesting")]:
        rc, msg = _open_rc(_blob_dir(tmp_path, raw, text))
        assert rc == ltxb.ELAYOUT and "manifest" in msg, (what, rc, msg)
    assert ltxb.lib.ltxb_blob_open(b"x", 4, ctypes.byref(ctypes.c_void_p())) == ltxb.EINVAL


def test_native_manifest_parser_details(tmp_path):
    """JSON the reference's parser accepts: escapes and non-ASCII in names,
    unknown fields (any type, nested, exponent numbers) ignored, other dtypes
    read as -1."""
    import ltxb
    data = bytes(range(64)) + bytes(8)
    man = {"packer_version": 1, "x": {"nested": [1, 2.5e3, None, True, {"y": "z"}]}, "align": 64,
           "block": -7, "total_bytes": 72, "blob_sha256": "",
           "entries": [{"name": "a.b\"c\\u00e9\U0001F600", "dtype": "BF16", "shape": [32], "offset": 0,
                        "nbytes": 64, "sha256": "", "extra": [[]]},
                       {"name": "tail", "dtype": "F16", "shape": [2, 2], "offset": 64, "nbytes": 8}]}
    d = _blob_dir(tmp_path, data, json.dumps(man, ensure_ascii=True))
    h = ctypes.c_void_p()
    assert ltxb.lib.ltxb_blob_open(d, 0, ctypes.byref(h)) == 0, ltxb.last_error()
    try:
        _, nb, ents, al, blk = _view(ltxb.lib, h)
        assert (nb, al, blk) == (72, 64, -7)
        assert ents[0].name.decode("utf-8") == man["entries"][0]["name"]
        assert ents[1].dtype == -1 and ents[1].ndim == 2 and list(ents[1].shape) == [2, 2]
    finally:
        ltxb.lib.ltxb_blob_close(h)


def test_blob_view_outlives_the_blob_object():
    """Blob.open's bytes stay mapped while any view of them is alive."""
    import gc

    import ltxb
    data = ltxb.Blob.open(GOLD, verify_digest=True, verify_entries=True).data
    gc.collect()
    assert bytes(data[:4096]) == (GOLD / "blob.bin").read_bytes()[:4096]


def test_layout_check_rejects_entries_past_the_end():
    """An entry whose offset + nbytes runs past the blob (or wraps a 64-bit
    sum back into range) is a layout error, never a later out-of-bounds
    read."""
    import ltxb
    names = [ctypes.c_char_p(n) for n in (b"a", b"b", b"c")]
    arr = (ltxb._Entry * 3)()
    for e, nm in zip(arr, names):
        e.name, e.dtype, e.ndim = nm, 1, 1
    arr[0].offset, arr[0].nbytes = 0, 64
    arr[1].offset, arr[1].nbytes = 64, (1 << 64) - 64   # 64 + nbytes wraps to 0
    arr[2].offset, arr[2].nbytes = 0, 128
    assert ltxb.lib.ltxb_blob_check_layout(ctypes.addressof(arr), 3, 128, 64) == ltxb.ELAYOUT
    assert "ends past the blob" in ltxb.last_error()
    arr[1].nbytes = 128                                   # 64 + 128 > 128
    assert ltxb.lib.ltxb_blob_check_layout(ctypes.addressof(arr), 2, 128, 64) == ltxb.ELAYOUT


@pytest.mark.parametrize("offset,nbytes", [((1 << 64) - 8, 64), (0, (1 << 64) - 1), (64, 128)])
def test_upload_rejects_entries_past_the_blob_before_any_device_call(offset, nbytes):
    """ltxb_weights_upload and ltxb_core_upload take caller-built entry tables.
    An entry whose offset + nbytes leaves the blob, including one whose 64-bit
    sum wraps back into range (offset = 2^64 - 8), is ELAYOUT, decided on the
    host before any device call, so no copy ever reads outside the blob."""
    import ltxb
    blob = (ctypes.c_uint8 * 128)()
    arr = (ltxb._Entry * 1)()
    arr[0].name, arr[0].dtype, arr[0].ndim = b"transformer_blocks_0_attn1_to_q_weight", 1, 2
    arr[0].shape[0], arr[0].shape[1] = 4, 8
    arr[0].offset, arr[0].nbytes = offset, nbytes
    h = ctypes.c_void_p()
    rc = ltxb.lib.ltxb_weights_upload(0, ctypes.addressof(blob), 128, ctypes.addressof(arr), 1, 0, ltxb.MODE_BF16,
                                      0, 256, 256, ctypes.byref(h))
    assert rc == ltxb.ELAYOUT, ltxb.last_error()
    assert "past the 128-byte blob" in ltxb.last_error()
    assert not h.value
    rc = ltxb.lib.ltxb_core_upload(0, ctypes.addressof(blob), 128, ctypes.addressof(arr), 1, 256, ctypes.byref(h))
    assert rc == ltxb.ELAYOUT, ltxb.last_error()
