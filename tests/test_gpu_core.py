"""GPU tests of the device-side steps either side of the block (the
reference's core parts, scheduler and RoPE tables), through the C ABI,
against the oracle's restatements."""

import numpy as np
import pytest
import torch

from oracle import blob as oblob
from oracle import core_ref as cr
from oracle import inputs as oin
from oracle import ltx_block_ref as ref

pytestmark = pytest.mark.gpu


def _ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in units in the last place of f32 (monotonic integer map)."""
    ia = a.astype(np.float32).view(np.int32).astype(np.int64)
    ib = b.astype(np.float32).view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


def _gate(got: np.ndarray, want: np.ndarray) -> None:
    """The reference's RoPE gate (ltx/block_conformance.zig:129-142): at most
    0.01 % of the values differ, each by at most one f32 ulp."""
    d = _ulp_diff(got, want)
    assert d.max() <= 1, f"worst {d.max()} ulp"
    assert (d != 0).sum() <= d.size // 10000, f"{(d != 0).sum()} stragglers of {d.size}"


@pytest.mark.parametrize("grid,H", [((22, 32, 40), 32), ((3, 5, 7), 32), ((4, 4, 4), 8)])
def test_rope_ltx_tables(cuda, grid, H):
    import ltxb
    pos = oin.grid_positions(*grid)
    rng = np.random.default_rng(0)
    # (start, end) cells: integer starts with fractional extents, as patchified latents have
    g = np.stack([pos.T, pos.T + rng.uniform(0.5, 1.5, size=pos.T.shape)], axis=-1).astype(np.float32)
    want_c, want_s = oin.rope_ltx(g, H * 128, H)
    cos, sin = ltxb.rope_tables(ltxb.ROPE_LTX, torch.from_numpy(g).to(cuda), H)
    torch.cuda.synchronize()
    _gate(cos.cpu().numpy(), want_c)
    _gate(sin.cpu().numpy(), want_s)
    assert (cos[:, 0, :2] == 1).all() and (sin[:, 0, :2] == 0).all()


@pytest.mark.parametrize("grid,H", [((22, 32, 40), 32), ((8, 8, 16), 4)])
def test_rope_axes_tables(cuda, grid, H):
    import ltxb
    pos = oin.grid_positions(*grid)
    want_c, want_s = oin.rope_axes(pos, H)
    cos, sin = ltxb.rope_tables(ltxb.ROPE_AXES, torch.from_numpy(pos.astype(np.float32)).to(cuda), H)
    torch.cuda.synchronize()
    _gate(cos.cpu().numpy(), want_c)
    _gate(sin.cpu().numpy(), want_s)


def test_rope_errors(cuda):
    import ltxb
    g = torch.zeros(3, 8, 2, device=cuda)
    with pytest.raises(ltxb.LtxbError):
        ltxb.rope_tables(7, g, 4)
    with pytest.raises(ltxb.LtxbError):
        ltxb.rope_tables(ltxb.ROPE_LTX, g, 64)  # more frequencies than the LTX layout has


# ---------------------------------------------------------------------------
# core parts
# ---------------------------------------------------------------------------

def _core(d, seed, device="cuda:0"):
    import ltxb
    cw = cr.make_core_weights(d, seed)
    data, entries = oblob.pack(cr.core_tensors(cw))
    ent = [dict(name=e.name, dtype=e.dtype, shape=e.shape, offset=e.offset, nbytes=e.nbytes) for e in entries]
    return cw, ltxb.Core(ltxb.Blob.from_bytes(data, ent), hidden=d)


def test_core_sinusoid(cuda):
    """The reference's sinusoid gate: both sides f32, rel-RMS <= 1e-5
    (ltx/core_conformance.zig:144-147)."""
    import ltxb
    t = np.concatenate([np.linspace(0, 1, 61), [0.909375, 0.725, 0.421875]]).astype(np.float32)
    got = ltxb.Core.sinusoid(torch.from_numpy(t).to(cuda)).cpu().numpy()
    assert ref.rel_rms(got, oin.sinusoid_f32(t)) <= 1e-5


@pytest.mark.parametrize("d", [256, 4096])
def test_core_adaln_pts2_patchify_tail(cuda, d):
    cw, core = _core(d, 11)
    oc = cr.CoreParts(cw)
    rng = np.random.default_rng(d)
    t = np.array([1.0, 0.725, 0.0], dtype=np.float32)
    emb, ts9 = core.adaln(torch.from_numpy(t).to(cuda))
    pts2 = core.pts2(torch.tensor([0.909375], device=cuda))
    T = 300
    lat = rng.standard_normal((T, 128)).astype(np.float32)
    x = core.patchify(torch.from_numpy(lat).to(cuda))
    xs = (rng.standard_normal((T, d)) * 2 + 0.3).astype(np.float32)
    tidx = rng.integers(0, 3, T).astype(np.int32)
    vel = core.tail(torch.from_numpy(xs).to(cuda), emb, torch.from_numpy(tidx).to(cuda))
    vel_tok = core.tail(torch.from_numpy(xs).to(cuda), emb[torch.from_numpy(tidx).long().to(cuda)].contiguous())
    torch.cuda.synchronize()
    want_emb = oc.emb(t)
    # f32 on the device vs f64; the reference's own gates are 2e-3 (ltx/core_conformance.zig:148-156)
    assert ref.rel_rms(emb.cpu().double(), want_emb) < 1e-4
    assert ref.rel_rms(ts9.cpu().double(), oc.ts9r(t)) < 1e-4
    assert ref.rel_rms(pts2.cpu().double(), oc.pts2r(0.909375)) < 1e-4
    assert ref.rel_rms(x.cpu().double(), oc.patchify(torch.from_numpy(lat).double())) < 1e-5
    want_vel = oc.tail_from_emb(torch.from_numpy(xs).double(), emb.cpu().double()[torch.from_numpy(tidx).long()])
    assert ref.rel_rms(vel.cpu().double(), want_vel) < 1e-5
    assert torch.equal(vel, vel_tok)
    # indices outside [0, K) read row 0, as the block's table select does
    bad = tidx.copy()
    bad[::4] = -1
    bad[1::9] = 3
    bad[2::10] = 2**31 - 1
    vel_bad = core.tail(torch.from_numpy(xs).to(cuda), emb, torch.from_numpy(bad).to(cuda))
    vel_zero = core.tail(torch.from_numpy(xs).to(cuda), emb,
                         torch.from_numpy(np.where((bad >= 0) & (bad < 3), bad, 0).astype(np.int32)).to(cuda))
    assert torch.equal(vel_bad, vel_zero)
    core.free()


def test_core_upload_errors(cuda):
    import ltxb
    cw = cr.make_core_weights(256, 0)
    tensors = [t for t in cr.core_tensors(cw) if not t[0].startswith("proj_out.bias")]
    data, entries = oblob.pack(tensors)
    ent = [dict(name=e.name, dtype=e.dtype, shape=e.shape, offset=e.offset, nbytes=e.nbytes) for e in entries]
    with pytest.raises(ltxb.LtxbError) as ei:
        ltxb.Core(ltxb.Blob.from_bytes(data, ent), hidden=256)
    assert ei.value.code == ltxb.EMISSING
    data, entries = oblob.pack(cr.core_tensors(cw))
    ent = [dict(name=e.name, dtype=e.dtype, shape=e.shape, offset=e.offset, nbytes=e.nbytes) for e in entries]
    with pytest.raises(ltxb.LtxbError) as ei:
        ltxb.Core(ltxb.Blob.from_bytes(data, ent), hidden=512)
    assert ei.value.code == ltxb.EDTYPE


# ---------------------------------------------------------------------------
# scheduler (bit-exact)
# ---------------------------------------------------------------------------

def test_scheduler_bit_exact(cuda):
    import ltxb
    rng = np.random.default_rng(7)
    T, C = 1000, 128
    clean = rng.standard_normal((T, C)).astype(np.float32)
    noise = rng.standard_normal((T, C)).astype(np.float32)
    mask = rng.choice(np.array([0.0, 0.5, 1.0, 0.3], dtype=np.float32), T)
    g = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    sig1 = ltxb.sched_sigmas(1)
    for scale in (1.0, 0.909375, 0.25):
        got = ltxb.sched_noise_init(g(clean), g(noise), g(mask), scale).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), cr.noise_init(clean, noise, mask, scale).view(np.uint32)), scale
    x = cr.noise_init(clean, noise, mask, 1.0)
    for i in range(len(sig1) - 1):
        s, sn = float(sig1[i]), float(sig1[i + 1])
        ts = ltxb.sched_timesteps(g(mask), s).cpu().numpy()
        assert np.array_equal(ts.view(np.uint32), cr.timesteps(mask, s).view(np.uint32))
        vel = rng.standard_normal((T, C)).astype(np.float32)
        got = ltxb.sched_step(g(x), g(vel), g(ts), g(clean), g(mask), s, sn).cpu().numpy()
        want = cr.scheduler_step(x, vel, ts, clean, mask, s, sn)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"step {i}"
        x = want


# ---------------------------------------------------------------------------
# the denoising loop
# ---------------------------------------------------------------------------

import helpers


@pytest.mark.parametrize("mode", ["f32", "int8"])
def test_denoise_loop_matches_oracle_trajectory(cuda, mode):
    """Three distilled steps over two blocks at D 256 (ltx/e2e_denoise.zig's
    loop): the latent after each step against the oracle's trajectory (core
    parts and blocks in f64, scheduler bit-exact f32). f32 blocks: rel-RMS
    1e-5. int8 blocks: the reference's per-step 2e-3 gate
    (ltx/e2e_denoise.zig:310-333), or the error of the same loop with the
    blocks in torch bf16 where that floor is higher."""
    import ltxb
    d, ff, grid = 256, 512, (2, 4, 8)
    T = grid[0] * grid[1] * grid[2]
    quant = "int8" if mode == "int8" else None
    blocks_o, blocks_g, bws = [], [], []
    for i in range(2):
        geom, bw, data, ent, qset = helpers.weights_case(d, ff, 20 + i, quant)
        bws.append((bw, qset))
        blocks_o.append(ref.QBlock(bw, torch.float64, qset=qset) if quant else ref.Block(bw, torch.float64))
        blocks_g.append(helpers.upload(data, ent, geom, ltxb.MODE_INT8 if quant else ltxb.MODE_F32))
    cw, core = _core(d, 5)
    inp = helpers.inputs_case(d, grid, 16, 4, "axes", 1, "random")
    rng = np.random.default_rng(9)
    clean = rng.standard_normal((T, 128)).astype(np.float32)
    noise = rng.standard_normal((T, 128)).astype(np.float32)
    mask_values = np.array([1.0, 0.5], dtype=np.float32)
    tidx = (np.arange(T) % 7 == 0).astype(np.int32)   # a few half-denoised tokens
    mask = mask_values[tidx]
    lat0 = cr.noise_init(clean, noise, mask, 1.0)
    sig = ltxb.sched_sigmas(1)[:4]
    want = cr.denoise_ref(cr.CoreParts(cw), blocks_o, sig, lat0, clean, mask, mask_values, tidx, inp.ctx,
                          inp.cos, inp.sin)
    g = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    got = []
    lat = g(lat0)
    for s in range(3):
        ltxb.denoise(core, blocks_g, sig[s:s + 2], lat, g(clean), g(mask), g(mask_values), g(tidx), g(inp.ctx),
                     g(inp.cos), g(inp.sin))
        got.append(lat.cpu().numpy().copy())
    lat_all = g(lat0)
    ltxb.denoise(core, blocks_g, sig, lat_all, g(clean), g(mask), g(mask_values), g(tidx), g(inp.ctx), g(inp.cos),
                 g(inp.sin))
    torch.cuda.synchronize()
    assert ltxb.device_status() == ltxb.OK
    if mode == "f32":
        tol = [1e-5] * 3
    else:
        # the bf16 deployment floor: the same loop with the blocks run in torch bf16
        b16_blocks = [ref.QBlock(bw, torch.bfloat16, qset=qs) for bw, qs in bws]
        b16 = cr.denoise_ref(cr.CoreParts(cw), b16_blocks, sig, lat0, clean, mask, mask_values, tidx, inp.ctx,
                             inp.cos, inp.sin, dtype=torch.bfloat16)
        tol = [max(2e-3, ref.rel_rms(b16[s], want[s])) for s in range(3)]
    for s in range(3):
        assert ref.rel_rms(got[s], want[s]) <= tol[s], (s, ref.rel_rms(got[s], want[s]), tol[s])
    assert np.array_equal(lat_all.cpu().numpy(), got[-1])  # one 3-step call == three 1-step calls
