"""GPU parity tests of the whole block through the C ABI, stage by stage, in
the reference's three precisions (ltx/block_conformance.zig's fence):

* f32 mode (reference `Block`): every stage within rel-RMS 1e-5 of the f64
  oracle -- BASELINE config 0 at full width (D 4096, T 1024, S 128).
* bf16 mode and int8 mode (reference `QBlock`, same dequantised weights in the
  oracle): rel-RMS <= 5e-3 and no worse than a torch-bf16 run of the same
  block (the reference's own "bf16 deployment floor",
  tools/make_oracle_bundle.py:184-200).
"""

import numpy as np
import pytest
import torch

import helpers
from oracle import ltx_block_ref as ref

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
LOW_TOL = 5e-3


def _run_stages(w, inp_t, stages):
    import ltxb
    blk = ltxb.Block(w)
    out = {}
    for s in stages:
        out[s] = blk.stage(s, *inp_t).double().cpu().numpy()
    torch.cuda.synchronize()
    assert ltxb.device_status() == ltxb.OK
    return out


def _check(got, want, tol, label):
    worst = {}
    for s, g in got.items():
        assert np.isfinite(g).all(), f"{label}/{s}: non-finite values"
        worst[s] = ref.rel_rms(g, want[s])
    bad = {s: e for s, e in worst.items() if e > tol}
    assert not bad, f"{label}: rel-RMS over {tol}: {bad} (all: {worst})"
    return worst


SMALL = dict(d=256, ff=512, grid=(2, 4, 16), s=16)


@pytest.mark.parametrize("adaln,k_rows,rope", [("random", 3, "axes"), ("mlp", 1, "ltx")])
def test_f32_small_all_stages(cuda, adaln, k_rows, rope):
    import ltxb
    geom, bw, data, ent, _ = helpers.weights_case(SMALL["d"], SMALL["ff"], 0, None)
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 0, rope, k_rows, adaln)
    want = helpers.oracle_stages(bw, inp)
    w = helpers.upload(data, ent, geom, ltxb.MODE_F32)
    got = _run_stages(w, helpers.to_cuda(inp, cuda), ref.STAGES)
    _check(got, want, F32_TOL, "f32-small")


def test_f32_config0(cuda):
    """D 4096, 32x128 heads, T 1024 on 8x8x16, S 128, FFN
    16384, RoPE 44/42/42, timestep 0.5 through the adaln MLP."""
    import ltxb
    geom, bw, data, ent, _ = helpers.weights_case(4096, 16384, 0, None)
    inp = helpers.inputs_case(4096, (8, 8, 16), 128, 0)
    want = helpers.oracle_stages(bw, inp)
    w = helpers.upload(data, ent, geom, ltxb.MODE_F32)
    got = _run_stages(w, helpers.to_cuda(inp, cuda), ref.STAGES)
    _check(got, want, F32_TOL, "f32-config0")
    w.free()


def _bf16_floor(bw, inp, qset=None):
    """The block run in torch bfloat16 on CPU (weights, inputs and every op in
    bf16), compared with f64: the reference's bf16 path analogue."""
    want = helpers.oracle_stages(bw, inp, qset)["block_out"]
    b16 = helpers.oracle_stages(bw, inp, qset, dtype=torch.bfloat16)["block_out"]
    return ref.rel_rms(b16, want)


@pytest.mark.parametrize("mode", ["bf16", "int8", "int8-ext-bf16scale"])
def test_lowp_small_all_stages(cuda, mode):
    import ltxb
    quant = None if mode == "bf16" else "int8"
    sdt = "bf16" if "bf16scale" in mode else "f32"
    qext = "ext" in mode
    geom, bw, data, ent, qset = helpers.weights_case(SMALL["d"], SMALL["ff"], 1, quant, sdt, qext)
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 1, "axes", 3, "random")
    oq = qset if quant else None
    want = helpers.oracle_stages(bw, inp, oq)
    w = helpers.upload(data, ent, geom, ltxb.MODE_BF16 if quant is None else ltxb.MODE_INT8, qext)
    got = _run_stages(w, helpers.to_cuda(inp, cuda), ref.STAGES)
    worst = _check(got, want, LOW_TOL, mode)
    floor = _bf16_floor(bw, inp, oq)
    assert worst["block_out"] <= max(floor, 1e-4), f"{mode}: {worst['block_out']} worse than torch-bf16 {floor}"


def test_qblockout_qkv_set(cuda):
    """QBlock.qBlockOut (ltx/block.zig:577-611): int8 q/k/v of both
    attentions with the FFN unquantised (QSET_QKV). Every stage within the
    low-precision bar of the oracle on the same dequantised q/k/v and no
    worse than torch-bf16; qBlockOut is the block call; a handle of the
    wrong set refuses the other method."""
    import ltxb
    geom, bw, data, ent, _ = helpers.weights_case(SMALL["d"], SMALL["ff"], 1, "int8")
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 1, "axes", 3, "random")
    want = helpers.oracle_stages(bw, inp, ref.Q8_FIELDS_QKV)
    w = ltxb.build_quant_bufs(ltxb.Blob.from_bytes(data, ent), 0, qset=ltxb.QSET_QKV, hidden=geom.d, ff=geom.ff)
    got = _run_stages(w, helpers.to_cuda(inp, cuda), ref.STAGES)
    worst = _check(got, want, LOW_TOL, "int8-qkv")
    floor = _bf16_floor(bw, inp, ref.Q8_FIELDS_QKV)
    assert worst["block_out"] <= max(floor, 1e-4), f"{worst['block_out']} worse than torch-bf16 {floor}"
    q = ltxb.QBlock(w)
    out = q.qBlockOut(*helpers.to_cuda(inp, cuda))
    assert np.array_equal(out.double().cpu().numpy(), got["block_out"])
    with pytest.raises(ltxb.LtxbError):
        q.qBlockOutAll(*helpers.to_cuda(inp, cuda))
    w.free()


def test_chain_and_wattn1(cuda):
    """Chain (ltx/block.zig:434-455): three f32-mode blocks back to back,
    against the oracle's chain at the f32 bar, and bit-identical to the
    blockOut calls composed by hand; wChainB47 is the same function here.
    wAttn1 (ltx/block.zig:274-276) is s3Attn1's call."""
    import ltxb
    cases = [helpers.weights_case(SMALL["d"], SMALL["ff"], 30 + i, None) for i in range(3)]
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 3, "axes", 3, "random")
    ws = [helpers.upload(data, ent, geom, ltxb.MODE_F32) for geom, _, data, ent, _ in cases]
    blocks = [ltxb.Block(w) for w in ws]
    chain = ltxb.Chain(*blocks)
    a = helpers.to_cuda(inp, cuda)
    c23 = chain.chainB23(*a)
    c47 = chain.chainB47(*a)
    w47 = chain.wChainB47(*a)
    by_hand = blocks[2].blockOut(blocks[1].blockOut(blocks[0].blockOut(*a), *a[1:]), *a[1:])
    torch.cuda.synchronize()
    assert torch.equal(c47, by_hand) and torch.equal(w47, c47)
    t = inp.torch()
    ob = [ref.Block(bw) for _, bw, _, _, _ in cases]
    y23 = ob[1].block_out(ob[0].block_out(*t), *t[1:])
    y47 = ob[2].block_out(y23, *t[1:])
    assert ref.rel_rms(c23.double().cpu().numpy(), y23) <= F32_TOL
    assert ref.rel_rms(c47.double().cpu().numpy(), y47) <= F32_TOL
    x, tstab, tidx, ctx, pts2, cos, sin = a
    assert torch.equal(blocks[0].wAttn1(x, tstab, tidx, cos, sin), blocks[0].s3Attn1(*a))
    assert ltxb.device_status() == ltxb.OK
    for w in ws:
        w.free()


@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_out_of_range_tidx_reads_row0(cuda, mode):
    """tidx entries outside [0, K) (negative, K, far above) select table row
    0, as the reference's select chain does (ltx/block.zig:47-67): every
    stage is bit-identical to the run with those entries set to 0 and matches
    the oracle's chain semantics. Every consumer of tidx (the norm-modulate
    rows and the gated-residual epilogues) is covered by the stage list."""
    import dataclasses
    import ltxb
    quant = None if mode == "f32" else "int8"
    geom, bw, data, ent, qset = helpers.weights_case(SMALL["d"], SMALL["ff"], 2, quant)
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 2, "axes", 3, "random")
    bad = inp.tidx.copy()
    bad[::5] = -1
    bad[1::7] = 3
    bad[2::11] = 2**31 - 1
    bad[3::13] = -2**31
    zeroed = np.where((bad >= 0) & (bad < 3), bad, 0).astype(np.int32)
    inp_bad = dataclasses.replace(inp, tidx=bad)
    w = helpers.upload(data, ent, geom, ltxb.MODE_F32 if quant is None else ltxb.MODE_INT8)
    got = _run_stages(w, helpers.to_cuda(inp_bad, cuda), ref.STAGES)
    same = _run_stages(w, helpers.to_cuda(dataclasses.replace(inp, tidx=zeroed), cuda), ref.STAGES)
    for s in ref.STAGES:
        assert np.array_equal(got[s], same[s]), f"{mode}/{s}: out-of-range tidx differs from row 0"
    want = helpers.oracle_stages(bw, inp_bad, qset if quant else None)
    _check(got, want, F32_TOL if quant is None else LOW_TOL, f"{mode}-tidx-oob")
    w.free()


@pytest.mark.parametrize("mode", ["bf16", "int8"])
def test_lowp_config0(cuda, mode):
    """Config-0 architecture at T = 1024 in bf16 / int8 (config 3's recipe:
    outliers, g128, f32 scales), block output and the conformance stages."""
    import ltxb
    quant = None if mode == "bf16" else "int8"
    geom, bw, data, ent, qset = helpers.weights_case(4096, 16384, 0, quant)
    inp = helpers.inputs_case(4096, (8, 8, 16), 128, 0)
    oq = qset if quant else None
    want = helpers.oracle_stages(bw, inp, oq)
    w = helpers.upload(data, ent, geom, ltxb.MODE_BF16 if quant is None else ltxb.MODE_INT8)
    got = _run_stages(w, helpers.to_cuda(inp, cuda), ref.STAGES)
    worst = _check(got, want, LOW_TOL, f"{mode}-config0")
    floor = _bf16_floor(bw, inp, oq)
    assert worst["block_out"] <= floor, f"{mode}: {worst['block_out']} worse than torch-bf16 {floor}"
    w.free()


def test_block_forward_deterministic_and_aliasing(cuda):
    import ltxb
    geom, bw, data, ent, _ = helpers.weights_case(SMALL["d"], SMALL["ff"], 2, "int8")
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 2, "axes", 3, "random")
    w = helpers.upload(data, ent, geom, ltxb.MODE_INT8)
    blk = ltxb.QBlock(w)
    t = helpers.to_cuda(inp, cuda)
    a = blk.qBlockOutAll(*t)
    b = blk.qBlockOutAll(*t)
    x2 = t[0].clone()
    blk.forward(x2, *t[1:], out=x2)  # out aliases x
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(a, x2)


def test_upload_errors(cuda):
    import ltxb
    geom, bw, data, ent, _ = helpers.weights_case(SMALL["d"], SMALL["ff"], 0, None)
    # int8 mode on a blob without ::q8 companions -> MissingEntry
    with pytest.raises(ltxb.LtxbError) as ei:
        helpers.upload(data, ent, geom, ltxb.MODE_INT8)
    assert ei.value.code == ltxb.EMISSING
    # wrong geometry -> dtype/shape error
    with pytest.raises(ltxb.LtxbError) as ei:
        ltxb.build_block_bufs(ltxb.Blob.from_bytes(data, ent), 0, hidden=512, ff=512)
    assert ei.value.code == ltxb.EDTYPE
    # mode mismatch between weights and config
    w = helpers.upload(data, ent, geom, ltxb.MODE_BF16)
    blk = ltxb.Block(w)
    blk.w.mode = ltxb.MODE_F32
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 0, "axes", 3, "random")
    with pytest.raises(ltxb.LtxbError):
        blk.forward(*helpers.to_cuda(inp, cuda))


def test_host_pipe_matches_device_forward(cuda):
    """ltxb_block_forward_host: pipelined host-buffer calls give exactly the
    device-buffer results, call by call (double-buffered staging reused)."""
    import ltxb
    geom, bw, data, ent, _ = helpers.weights_case(SMALL["d"], SMALL["ff"], 2, "int8")
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 2, "axes", 3, "random")
    w = helpers.upload(data, ent, geom, ltxb.MODE_INT8)
    blk = ltxb.QBlock(w)
    x, tstab, tidx, ctx, pts2, cos, sin = helpers.to_cuda(inp, cuda)
    pipe = blk.host_pipe(tstab, tidx, ctx, pts2, cos, sin, x.shape[0])
    xs = [(x.cpu() * (1.0 + 0.25 * i)).pin_memory() for i in range(5)]
    outs = [torch.empty_like(xs[0]).pin_memory() for _ in xs]
    for xi, oi in zip(xs, outs):
        pipe.forward(xi, oi)
    pipe.join()
    torch.cuda.synchronize()
    for xi, oi in zip(xs, outs):
        want = blk.forward(xi.to(cuda), tstab, tidx, ctx, pts2, cos, sin)
        torch.cuda.synchronize()
        assert torch.equal(oi, want.cpu())
    pipe.free()


def test_workspace_is_not_overrun(cuda):
    """The block stays inside ltxb_block_workspace_bytes: a guard region
    after the workspace is untouched (int8 with FF < 3 D, where the fused
    q/k/v matrix is the largest one expanded)."""
    import ltxb
    geom, bw, data, ent, _ = helpers.weights_case(SMALL["d"], SMALL["ff"], 2, "int8")
    inp = helpers.inputs_case(SMALL["d"], SMALL["grid"], SMALL["s"], 2, "axes", 3, "random")
    w = helpers.upload(data, ent, geom, ltxb.MODE_INT8)
    blk = ltxb.QBlock(w)
    t = helpers.to_cuda(inp, cuda)
    need = blk.workspace_bytes(t[0].shape[0], t[3].shape[0], t[1].shape[0])
    guard = 1 << 20
    blk._ws = torch.full((need + 256 + guard,), 0xA5, dtype=torch.uint8, device=cuda)
    start = ((blk._ws.data_ptr() + 255) & ~255) - blk._ws.data_ptr()
    blk.forward(*t)
    torch.cuda.synchronize()
    assert bool((blk._ws[start + need:] == 0xA5).all())
