"""CPU tests of the core-parts / scheduler restatement (oracle/core_ref.py)
and of the host side of the library's scheduler (no GPU needed)."""

from fractions import Fraction

import numpy as np
import torch

from oracle import core_ref as cr
from oracle import ltx_block_ref as ref


def _round_f32_exact(t: Fraction) -> np.float32:
    """Correct round-to-nearest-even of a rational to f32."""
    f = np.float32(float(t))
    cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
    return min(cands, key=lambda x: (abs(Fraction(float(x)) - t), int(np.float32(x).view(np.int32)) & 1))


def test_fma32_is_correctly_rounded():
    rng = np.random.default_rng(0)
    a = rng.standard_normal(3000).astype(np.float32)
    b = rng.standard_normal(3000).astype(np.float32)
    c = (rng.standard_normal(3000) * np.exp2(rng.integers(-30, 30, 3000))).astype(np.float32)
    # plus exact-halfway constructions: a*b a power-of-two fraction of c's ulp
    a[:200] = np.float32(1.0)
    b[:200] = np.float32(2.0) ** -25
    c[:200] = np.float32(1.0) + np.arange(200, dtype=np.float32) * np.float32(2.0) ** -23
    got = cr.fma32(a, b, c)
    for i in range(0, 3000, 3):
        want = _round_f32_exact(Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i])))
        assert got[i] == want, i


def test_lerp_matches_torch():
    """torch.lerp on CPU is the reference's ground truth (ltx/scheduler.zig:20-35)."""
    rng = np.random.default_rng(1)
    x = rng.standard_normal(50000).astype(np.float32)
    y = rng.standard_normal(50000).astype(np.float32)
    for w in (0.0, 0.3, 0.4999, 0.5, 0.909375, 1.0, -0.2):
        want = torch.lerp(torch.from_numpy(x), torch.from_numpy(y), float(np.float32(w))).numpy()
        assert np.array_equal(cr.lerp(x, y, np.float32(w)), want), w


def test_scheduler_semantics():
    """Euler with no sigma = 0 special case; noise init at scale 1 and mask 1
    returns the noise; timesteps are mask * sigma."""
    rng = np.random.default_rng(2)
    T, C = 64, 128
    x = rng.standard_normal((T, C)).astype(np.float32)
    clean = rng.standard_normal((T, C)).astype(np.float32)
    noise = rng.standard_normal((T, C)).astype(np.float32)
    mask = np.ones(T, dtype=np.float32)
    assert np.array_equal(cr.noise_init(clean, noise, mask, 1.0), noise)
    ts = cr.timesteps(mask, 0.725)
    assert ts.dtype == np.float32 and (ts == np.float32(0.725)).all()
    vel = rng.standard_normal((T, C)).astype(np.float32)
    out = cr.scheduler_step(x, vel, ts, clean, mask, 0.421875, 0.0)
    den = cr.post_process(cr.to_denoised(x, vel, ts), clean, mask)
    assert np.abs(out - den).max() < 1e-5  # the last step lands on `denoised` up to rounding


def test_library_sigmas_match_reference_lists():
    import ltxb
    assert np.array_equal(ltxb.sched_sigmas(1).view(np.uint32), cr.SIGMAS_STAGE1.view(np.uint32))
    assert np.array_equal(ltxb.sched_sigmas(2).view(np.uint32), cr.SIGMAS_STAGE2.view(np.uint32))


def test_tail_norm_kind_has_teeth():
    """ltx/core_conformance.zig:195-212: the tail with RMSNorm in place of
    LayerNorm must miss the true tail by more than 1e-3 rel-RMS."""
    cw = cr.make_core_weights(256, seed=3)
    core = cr.CoreParts(cw)
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((32, 256)) + 0.5)
    e = core.emb(np.full(32, 0.7, dtype=np.float32))
    good = core.tail_from_emb(x, e)
    wrong = ref.lin(ref.modulate(ref.rms_no_w(x), cw.t["fsst"][1] + e, cw.t["fsst"][0] + e), cw.t["po_w"], cw.t["po_b"])
    assert ref.rel_rms(wrong, good) > 1e-3
