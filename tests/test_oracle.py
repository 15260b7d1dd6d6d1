"""CPU tests of the oracle itself: pinned against the golden vectors made by
the reference's own tools, and against the internal known-answer tests of the
reference's conformance suite (ltx/block_conformance.zig)."""

import json
import pathlib

import numpy as np
import pytest
import torch

from oracle import blob as oblob
from oracle import inputs as oin
from oracle import ltx_block_ref as ref

GOLD = pathlib.Path(__file__).resolve().parent / "golden" / "ref_tools"


def _bf16_file(name, shape):
    return np.frombuffer((GOLD / name).read_bytes(), dtype=np.uint16).reshape(shape)


def _manifest():
    return json.loads((GOLD / "manifest.json").read_text())


QUANT_SET = ["attn1.to_q.weight", "attn1.to_k.weight", "attn1.to_v.weight", "ff.net.0.proj.weight",
             "ff.net.2.weight"]


@pytest.mark.parametrize("name", QUANT_SET)
def test_quantiser_matches_reference_tool(name):
    """oracle.quantize_g128 == tools/quantize_block.py (int8, gs 128) bit for bit."""
    man = _manifest()
    e = man["tensors"][f"transformer_blocks.0.{name}"]
    stem = e["file"].removesuffix(".bin")
    w = ref.bf16_to_f32(_bf16_file(e["file"], e["shape"]))
    q, sc = ref.quantize_g128(w)
    gold_q = np.frombuffer((GOLD / f"{stem}_q8.bin").read_bytes(), dtype=np.int8).reshape(e["shape"])
    gold_s = np.frombuffer((GOLD / f"{stem}_q8scale.bin").read_bytes(), dtype=np.float32)
    gold_s = gold_s.reshape(e["shape"][0], e["shape"][1] // 128)
    assert np.array_equal(q, gold_q)
    assert np.array_equal(sc.view(np.uint32), gold_s.view(np.uint32))


def test_quantiser_edge_cases():
    """absmax == 0 rows/groups get scale 1.0 and q == 0 (tools/quantize_block.py:56)."""
    man = _manifest()
    e = man["tensors"]["transformer_blocks.0.attn1.to_q.weight"]
    stem = e["file"].removesuffix(".bin")
    gold_s = np.frombuffer((GOLD / f"{stem}_q8scale.bin").read_bytes(), dtype=np.float32).reshape(32, 2)
    gold_q = np.frombuffer((GOLD / f"{stem}_q8.bin").read_bytes(), dtype=np.int8).reshape(32, 256)
    assert (gold_s[3] == 1.0).all() and (gold_q[3] == 0).all()       # all-zero row
    assert gold_s[5, 0] == 1.0 and (gold_q[5, :128] == 0).all()      # all-zero group
    assert gold_q.min() >= -128 and gold_q.max() <= 127


def test_dequant_roundtrip_error():
    """KAT (4): quantiser round trip of N(0, 0.02) weights has rel-RMS ~0.007-0.013."""
    w = oin.normal_f32(0, "rt", (256, 1024), 0.02)
    q, sc = ref.quantize_g128(w)
    rel = ref.rel_rms(ref.dequant(q, sc), w)
    assert 0.003 < rel < 0.02


def test_bf16_scales_consistent():
    """bf16 scales: q is computed against the rounded scale."""
    w = oin.apply_outliers(oin.normal_f32(1, "bs", (64, 512), 0.02), 1, "bs")
    q, s16 = ref.quantize_g128(w, scale_dtype="bf16")
    assert s16.dtype == np.uint16
    deq = ref.dequant(q, s16)
    assert ref.rel_rms(deq, w) < 0.02
    assert np.abs(q).max() <= 128


def test_packer_matches_reference_tool():
    """oracle.blob.pack == tools/pack_block.py byte for byte (offsets, fill, order)."""
    man = _manifest()
    gold_blob = (GOLD / "blob.bin").read_bytes()
    gold_man = json.loads((GOLD / "blob_manifest.json").read_text())
    tensors = []
    for short, e in man["tensors"].items():
        tensors.append((short, e["dtype"], e["shape"], (GOLD / e["file"]).read_bytes()))
        stem = e["file"].removesuffix(".bin")
        if (GOLD / f"{stem}_q8.bin").exists():
            o, i = e["shape"]
            tensors.append((short + "::q8", "I8", [o, i], (GOLD / f"{stem}_q8.bin").read_bytes()))
            tensors.append((short + "::q8scale", "F32", [o, i // 128], (GOLD / f"{stem}_q8scale.bin").read_bytes()))
    data, entries = oblob.pack(tensors)
    assert data == gold_blob
    assert [(e.name, e.offset, e.nbytes, e.sha256) for e in entries] == \
        [(e["name"], e["offset"], e["nbytes"], e["sha256"]) for e in gold_man["entries"]]
    oblob.check_layout(entries, len(data))


def test_layout_errors():
    """ltx/loader.zig:73-82 error names."""
    E = oblob.Entry
    with pytest.raises(ValueError, match="Misaligned"):
        oblob.check_layout([E("a", "I8", [1], 0, 10, ""), E("b", "I8", [1], 70, 10, "")], 80)
    with pytest.raises(ValueError, match="LayoutGap"):
        oblob.check_layout([E("a", "I8", [1], 0, 10, ""), E("b", "I8", [1], 128, 10, "")], 138)
    with pytest.raises(ValueError, match="TrailingBytes"):
        oblob.check_layout([E("a", "I8", [1], 0, 10, "")], 64)


def test_online_softmax_equals_dense():
    """KAT (3): whileSdpa == dense SDPA within 1e-5 at chunk 16 and 1024
    (ltx/block_conformance.zig:406)."""
    g = torch.Generator().manual_seed(0)
    for t, chunk in ((64, 16), (2048, 1024)):
        q = torch.randn(t, 2, 128, generator=g, dtype=torch.float64)
        k = torch.randn(t, 2, 128, generator=g, dtype=torch.float64)
        v = torch.randn(t, 2, 128, generator=g, dtype=torch.float64)
        dense = ref.sdpa_dense(q, k, v)
        wh = ref.while_sdpa_c(chunk, q, k, v)
        assert ref.rel_rms(wh, dense) < 1e-12
    # f32 agreement (the reference's gate is in f32)
    q32, k32, v32 = (torch.randn(256, 2, 128, generator=g) for _ in range(3))
    assert ref.rel_rms(ref.while_sdpa_c(16, q32, k32, v32), ref.sdpa_dense(q32, k32, v32)) < 1e-5


def test_rope_identity_slots():
    """KAT (1): LTX table head 0 slots 0, 1 are exactly (1, 0)
    (ltx/block_conformance.zig:155-163), and the frequency grid is f32-rounded."""
    pos = oin.grid_positions(4, 4, 4)
    g = np.stack([pos.T, pos.T], axis=-1).astype(np.float32)
    cos, sin = oin.rope_ltx(g, 4096, 32)
    assert cos.shape == (64, 32, 64)
    assert (cos[:, 0, :2] == 1.0).all() and (sin[:, 0, :2] == 0.0).all()
    ind = oin.ltx_freq_grid(682)
    assert np.array_equal(ind, ind.astype(np.float32).astype(np.float64))
    assert ind[0] == np.float64(np.float32(np.pi / 2))


def test_rope_axes_layout():
    """BASELINE 44/42/42 table: slot 0 / 22 / 43 rotate by the F / H / W index."""
    pos = oin.grid_positions(8, 8, 16)
    cos, sin = oin.rope_axes(pos, 4)
    t = 5 * 128 + 3 * 16 + 7
    assert np.isclose(np.arctan2(sin[t, 0, 0], cos[t, 0, 0]), 5.0 - 2 * np.pi)
    assert np.isclose(np.arctan2(sin[t, 2, 22], cos[t, 2, 22]), 3.0)
    assert np.isclose(np.arctan2(sin[t, 3, 43], cos[t, 3, 43]), 7.0 - 2 * np.pi)
    assert np.allclose(cos[:, 0], cos[:, 3])


def _small_case(seed=0, t_grid=(2, 4, 8), s=16, d=256, ff=512):
    geom = ref.Geometry(d=d, ff=ff)
    bw = oin.make_weights(geom, seed)
    inp = oin.make_inputs(geom, grid=t_grid, s=s, seed=seed, adaln="random", k_rows=3)
    return bw, inp


def test_staged_equals_oneshot():
    """KAT (2): the staged composition == the one-shot block (f64), and every
    prefix-recomputing stage method equals the one-pass stage dump."""
    bw, inp = _small_case()
    blk = ref.Block(bw)
    a = inp.torch()
    st = blk.staged(*a)
    x, tstab, tidx, ctx, pts2, cos, sin = a
    assert torch.equal(st["block_out"], blk.block_out(*a))
    assert torch.allclose(st["s1_norm_msa"], blk.s1_norm_msa(x, tstab, tidx), rtol=0, atol=0)
    assert torch.allclose(st["s4_after_sa"], blk.s4_after_sa(x, tstab, tidx, cos, sin), rtol=0, atol=0)
    assert torch.allclose(st["s6_ff_in"], blk.s6_ff_in(*a), rtol=0, atol=0)
    assert torch.allclose(st["s7_ff_out"], blk.s7_ff_out(*a), rtol=0, atol=0)
    assert ref.rel_rms(blk.w_block_out(*a), st["block_out"]) < 1e-12


def test_qblock_close_to_block():
    """KAT (5): the int8 block stays within the reference's 2e-2 quant budget
    of the bf16-weight block (ltx/block_conformance.zig:494)."""
    geom = ref.Geometry(d=256, ff=512)
    bw = oin.make_weights(geom, 0, quant="int8", outliers=False)
    inp = oin.make_inputs(geom, grid=(2, 4, 8), s=16, seed=0)
    a = inp.torch()
    full = ref.Block(bw).block_out(*a)
    q = ref.QBlock(bw).q_block_out_all(*a)
    assert 0 < ref.rel_rms(q, full) < 2e-2


def test_ada_gather_matches_select_chain():
    """ada_val gathers the same rows the reference's select-chain picks."""
    g = torch.Generator().manual_seed(3)
    tstab = torch.randn(3, 9, 8, generator=g, dtype=torch.float64)
    sst = torch.randn(9, 8, generator=g, dtype=torch.float64)
    tidx = torch.tensor([0, 2, 1, 1, 0, 2], dtype=torch.int32)
    got = ref.ada_val(sst, tstab, tidx, 4)
    tv = tstab[0, 4].expand(6, 8).clone()
    for k in range(1, 3):
        tv = torch.where((tidx == k)[:, None], tstab[k, 4].expand(6, 8), tv)
    assert torch.equal(got, tv + sst[4])


def test_ada_out_of_range_tidx_reads_row0():
    """An index the chain never matches (negative, K or above) keeps the
    chain's default, row 0, in the gather as in the chain itself."""
    g = torch.Generator().manual_seed(4)
    tstab = torch.randn(4, 9, 8, generator=g, dtype=torch.float64)
    sst = torch.randn(9, 8, generator=g, dtype=torch.float64)
    tidx = torch.tensor([3, -1, 4, 1, 2**31 - 1, 0, -2**31, 2, 7], dtype=torch.int32)
    got = ref.ada_val(sst, tstab, tidx, 5)
    assert torch.equal(got, ref.select_chain_rows(tstab[:, 5], tidx) + sst[5])
    clamped = torch.where((tidx >= 0) & (tidx < 4), tidx, torch.zeros_like(tidx))
    assert torch.equal(got, ref.ada_val(sst, tstab, clamped, 5))


def test_quant_probes_within_reference_budgets():
    """The reference's five quantisation probes (ltx/block_conformance.zig:
    488-494: qLogits 5e-2, qAttn1 2e-2, qBlockOut 2e-2, qFfOut 5e-2,
    qBlockOutAll 2e-2 against the unquantised block) on the oracle, int8 g128
    weights without outlier channels. Each probe must show a nonzero error
    (its linears really are quantised) inside its budget."""
    geom = ref.Geometry(d=256, ff=512)
    bw = oin.make_weights(geom, 0, quant="int8", outliers=False)
    inp = oin.make_inputs(geom, grid=(2, 4, 8), s=16, seed=0)
    probes = ref.quant_probes(bw, *inp.torch())
    assert [(f, q) for f, q, _, _ in probes] == [("fLogits", "qLogits"), ("s3Attn1", "qAttn1"),
                                                 ("blockOut", "qBlockOut"), ("s7FfOut", "qFfOut"),
                                                 ("blockOut", "qBlockOutAll")]
    for f, q, err, budget in probes:
        assert 0 < err < budget, (f, q, err, budget)


def test_logits_and_blockwise_attn1():
    """fLogits is q.k before the softmax: softmax(logits / sqrt(hd)) applied
    to v reproduces s2Attn1NoGate's attention core; wAttn1 (blockwise
    softmax) equals s3Attn1 (dense) to rounding (ltx/block_conformance.zig:
    391-406 gates them at 1e-5)."""
    geom = ref.Geometry(d=256, ff=512)
    bw = oin.make_weights(geom, 1)
    inp = oin.make_inputs(geom, grid=(2, 4, 8), s=16, seed=1)
    x, tstab, tidx, ctx, pts2, cos, sin = inp.torch()
    blk = ref.Block(bw)
    lg = blk.f_logits(x, tstab, tidx, cos, sin)
    t, h = x.shape[0], geom.h
    assert lg.shape == (t, h, t)
    n = blk.s1_norm_msa(x, tstab, tidx)
    v = ref.lin(n, blk.w["v1_w"], blk.w["v1_b"]).reshape(t, h, ref.HD)
    p = torch.softmax(lg / np.sqrt(ref.HD), dim=2)
    core = torch.einsum("qhk,khd->qhd", p, v).reshape(t, h * ref.HD)
    want = ref.lin(core, blk.w["o1_w"], blk.w["o1_b"])
    assert ref.rel_rms(want, blk.s2_attn1_nogate(x, tstab, tidx, cos, sin)) < 1e-12
    assert ref.rel_rms(blk.w_attn1(x, tstab, tidx, cos, sin), blk.s3_attn1(x, tstab, tidx, cos, sin)) < 1e-12


def test_staged_rows_equals_staged_on_those_rows():
    """The sampled-rows restatement used at full length equals the one-pass
    staged block on the same rows (K/V over all tokens, queries on the
    sample), in f64, on int8 EXT weights with bf16 scales."""
    geom = ref.Geometry(d=256, ff=512)
    bw = oin.make_weights(geom, 3, quant="int8", scale_dtype="bf16", qset=ref.Q8_FIELDS_EXT)
    inp = oin.make_inputs(geom, grid=(2, 4, 16), s=16, seed=3, adaln="random", k_rows=3)
    blk = ref.QBlock(bw, qset=ref.Q8_FIELDS_EXT)
    args = inp.torch()
    full = blk.staged(*args)
    rows = np.array([0, 5, 63, 64, 100, 127])
    part = blk.staged_rows(*args, rows=rows, head_group=1)
    for s in ref.STAGES:
        assert ref.rel_rms(part[s].numpy(), full[s][rows].numpy()) < 1e-12, s


def test_block_weights_read_back_from_a_blob():
    """oracle.blob.block_weights_from_blob inverts block_tensors + pack: the
    stored bytes come back exactly, and a quantised field stored without its
    bf16 original is its exact dequantisation."""
    from oracle import blob as oblob
    geom = ref.Geometry(d=256, ff=512)
    bw = oin.make_weights(geom, 4, quant="int8", scale_dtype="bf16", qset=ref.Q8_FIELDS_EXT)
    data, ent = oblob.pack(oblob.block_tensors(bw, 0))
    back = oblob.block_weights_from_blob(data, ent, geom)
    for k, v in bw.raw.items():
        assert np.array_equal(back.raw[k], v), k
    drop = {oblob.normalize_name("transformer_blocks.0." + oblob.DOTTED["o1_w"])}
    data2, ent2 = oblob.pack([t for t in oblob.block_tensors(bw, 0) if oblob.normalize_name(t[0]) not in drop])
    back2 = oblob.block_weights_from_blob(data2, ent2, geom)
    want = ref.dequant(bw.raw["o1_w::q8"], bw.raw["o1_w::q8scale"])
    assert np.array_equal(back2.t["o1_w"].numpy(), want)
