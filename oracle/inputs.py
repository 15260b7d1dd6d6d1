"""Seeded synthetic inputs for the BASELINE configs -- TEST INFRASTRUCTURE ONLY.

The same bytes feed both the CPU oracle and the GPU library (the GPU side gets
them through the C-ABI upload path), so parity compares like with like.

* weights: N(0, 0.02) drawn in f32 and stored as bf16 (the reference's
  checkpoint dtype, ltx/block.zig:377-406); q/k norm weights 1 + N(0, 0.02);
  `sst` [9, D] and `psst` [2, D] N(0, 0.02) kept f32.
* int8 linears: BASELINE config 2's recipe -- 0.5% of input channels scaled
  x20 (outliers), then symmetric grouped-128 quantisation
  (tools/quantize_block.py:52-59), scales f32 (reference) or bf16 (BASELINE).
* RoPE tables in two layouts:
  - "axes": BASELINE's head-dim split 44/42/42 over (F, H, W), theta 10000.
    Each head's 64 rotation slots: [0, 22) use frequencies theta^(-2i/44)
    times the frame index, [22, 43) theta^(-2i/42) times the row index,
    [43, 64) theta^(-2i/42) times the column index; identical for all heads.
  - "ltx": the reference's bands-across-heads table of
    ltx/block_conformance.zig:87-127 (frequency grid theta^linspace * pi/2
    rounded to f32, fractional positions 2*(mid/max_pos)-1, 2 prepended
    identity slots, slot j = h*64 + f -> frequency (j-2)/3, axis (j-2)%3).
* timestep modulation: ts9 / pts2 from core_parts' adaln MLPs
  (ltx/core_parts.zig:42-49, :115-128) with N(0, 0.02) weights at timestep
  0.5: sinusoid of t*1000 in f32 (cos half first), linear -> SiLU -> linear,
  then SiLU -> chunk linear; K = 1 row, tidx = 0.
"""

from __future__ import annotations

import math
import zlib
from dataclasses import dataclass

import numpy as np
import torch

from . import ltx_block_ref as ref

THETA = 10000.0
LTX_MAX_POS = (20.0, 2048.0, 2048.0)


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def normal_f32(seed: int, name: str, shape, std: float) -> np.ndarray:
    g = _rng(seed, name)
    return (g.standard_normal(size=shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def bf16_tensor(a: np.ndarray) -> tuple[np.ndarray, torch.Tensor]:
    """f32 array -> (bf16 bits uint16, exact float64 torch tensor)."""
    u = ref.bf16_round(a)
    return u, torch.from_numpy(ref.bf16_to_f32(u).astype(np.float64))


def make_weights(geom: ref.Geometry, seed: int = 0, quant: str | None = None,
                 scale_dtype: str = "f32", qset=ref.Q8_FIELDS, outliers: bool = True,
                 std: float = 0.02) -> ref.BlockWeights:
    """One block's weights per the spec in the module docstring.

    quant=None: every matrix bf16. quant="int8": fields in `qset` also get
    `::q8` / `::q8scale` companions (the bf16 original is kept too, as the
    reference blob keeps both, tools/pack_block.py:41-47)."""
    bw = ref.BlockWeights(geom=geom)
    for fname, _stem, dims in ref.WEIGHT_SPECS:
        shape = geom.dims(dims)
        if fname in ref.F32_FIELDS:
            a = normal_f32(seed, fname, shape, std)
            bw.raw[fname] = a
            bw.t[fname] = torch.from_numpy(a.astype(np.float64))
            continue
        a = normal_f32(seed, fname, shape, std)
        if fname.startswith(("qn", "kn")):
            a = (a + np.float32(1.0)).astype(np.float32)
        if quant == "int8" and fname in qset and outliers:
            a = apply_outliers(a, seed, fname)
        u, t = bf16_tensor(a)
        bw.raw[fname] = u
        bw.t[fname] = t
        if quant == "int8" and fname in qset:
            w = ref.bf16_to_f32(u)
            q, sc = ref.quantize_g128(w, scale_dtype=scale_dtype)
            bw.raw[fname + "::q8"] = q
            bw.raw[fname + "::q8scale"] = sc
    return bw


def apply_outliers(w: np.ndarray, seed: int, name: str, frac: float = 0.005, mult: float = 20.0) -> np.ndarray:
    """0.5% of input channels (the K axis) scaled x20."""
    k = w.shape[1]
    n_out = max(1, int(round(frac * k)))
    cols = _rng(seed, name + "/outliers").choice(k, size=n_out, replace=False)
    w = w.copy()
    w[:, cols] *= np.float32(mult)
    return w


# ---------------------------------------------------------------------------
# RoPE tables
# ---------------------------------------------------------------------------

def grid_positions(f: int, h: int, w: int) -> np.ndarray:
    """Integer (frame, row, col) per token, token order t = (fi*h + hi)*w + wi."""
    fi, hi, wi = np.meshgrid(np.arange(f), np.arange(h), np.arange(w), indexing="ij")
    return np.stack([fi.ravel(), hi.ravel(), wi.ravel()], axis=1).astype(np.float64)


def rope_axes(pos: np.ndarray, n_heads: int, split=(44, 42, 42), theta: float = THETA):
    """BASELINE layout (see module docstring). Returns cos, sin f32 [T, H, 64]."""
    assert sum(split) == 128
    ang = []
    for axis, dims in enumerate(split):
        npair = dims // 2
        inv = theta ** (-2.0 * np.arange(npair, dtype=np.float64) / dims)
        ang.append(pos[:, axis:axis + 1] * inv[None, :])
    a = np.concatenate(ang, axis=1)                              # [T, 64]
    cos = np.broadcast_to(np.cos(a)[:, None, :], (pos.shape[0], n_heads, 64))
    sin = np.broadcast_to(np.sin(a)[:, None, :], (pos.shape[0], n_heads, 64))
    return np.ascontiguousarray(cos, dtype=np.float32), np.ascontiguousarray(sin, dtype=np.float32)


def ltx_freq_grid(nf: int, theta: float = THETA) -> np.ndarray:
    """ltx/block_conformance.zig:93-99: theta^(k/(nf-1)) * pi/2 in f64,
    rounded to f32, promoted back to f64."""
    k = np.arange(nf, dtype=np.float64) / (nf - 1)
    return (np.power(theta, k) * (math.pi / 2.0)).astype(np.float32).astype(np.float64)


def rope_ltx(grid: np.ndarray, d: int, n_heads: int, theta: float = THETA,
             max_pos=LTX_MAX_POS):
    """ltx/block_conformance.zig:87-127. grid: [3, T, 2] (start, end) f32
    positions. Returns cos, sin f32 [T, H, 64] (the block's layout)."""
    nf = d // 6
    ind = ltx_freq_grid(nf, theta)
    t = grid.shape[1]
    mid = (grid[:, :, 0].astype(np.float64) + grid[:, :, 1].astype(np.float64)) / 2.0
    arg = (mid / np.asarray(max_pos, dtype=np.float64)[:, None]) * 2.0 - 1.0   # [3, T]
    j = np.arange(n_heads * 64)
    s = np.maximum(j - 2, 0)
    freq = ind[s // 3][None, :] * arg[s % 3].T                               # [T, H*64]
    c = np.cos(freq)
    sn = np.sin(freq)
    c[:, j < 2] = 1.0
    sn[:, j < 2] = 0.0
    cos = c.reshape(t, n_heads, 64).astype(np.float32)
    sin = sn.reshape(t, n_heads, 64).astype(np.float32)
    return cos, sin


# ---------------------------------------------------------------------------
# timestep modulation (core_parts)
# ---------------------------------------------------------------------------

def sinusoid_f32(t: np.ndarray) -> np.ndarray:
    """ltx/core_parts.zig:42-49: f32 sinusoid of t*1000, cos half first."""
    half = 128
    idx = np.arange(half, dtype=np.float32)
    freqs = np.exp(idx * np.float32(-math.log(1e4) / half)).astype(np.float32)
    arg = (t.astype(np.float32)[:, None] * np.float32(1000.0)) * freqs[None, :]
    return np.concatenate([np.cos(arg), np.sin(arg)], axis=1).astype(np.float32)


def _silu(x):
    return x * torch.sigmoid(x)


def adaln_tables(d: int, seed: int = 0, timestep: float = 0.5, sigma: float = 0.5, std: float = 0.02):
    """ts9 [1, 9, D] and pts2 [2, D] (f32) via the core_parts MLPs
    (ltx/core_parts.zig:115-141), f64 arithmetic after the f32 sinusoid."""
    def w(name, shape):
        return bf16_tensor(normal_f32(seed, name, shape, std))[1]
    sin_t = torch.from_numpy(sinusoid_f32(np.array([timestep])).astype(np.float64))
    e = ref.lin(_silu(ref.lin(sin_t, w("ada_l1_w", (d, 256)), w("ada_l1_b", (d,)))),
                w("ada_l2_w", (d, d)), w("ada_l2_b", (d,)))
    ts9 = ref.lin(_silu(e), w("ada_out_w", (9 * d, d)), w("ada_out_b", (9 * d,)))
    sin_s = torch.from_numpy(sinusoid_f32(np.array([sigma])).astype(np.float64))
    pe = ref.lin(_silu(ref.lin(sin_s, w("pada_l1_w", (d, 256)), w("pada_l1_b", (d,)))),
                 w("pada_l2_w", (d, d)), w("pada_l2_b", (d,)))
    pts2 = ref.lin(_silu(pe), w("pada_out_w", (2 * d, d)), w("pada_out_b", (2 * d,)))
    return (ts9.reshape(1, 9, d).numpy().astype(np.float32),
            pts2.reshape(2, d).numpy().astype(np.float32))


# ---------------------------------------------------------------------------
# block inputs
# ---------------------------------------------------------------------------

@dataclass
class BlockInputs:
    x: np.ndarray        # [T, D] f32
    tstab: np.ndarray    # [K, 9, D] f32
    tidx: np.ndarray     # [T] int32
    ctx: np.ndarray      # [S, D] f32
    pts2: np.ndarray     # [2, D] f32
    cos: np.ndarray      # [T, H, 64] f32
    sin: np.ndarray      # [T, H, 64] f32

    def torch(self, dtype=torch.float64):
        c = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dtype)
        return (c(self.x), c(self.tstab), torch.from_numpy(self.tidx), c(self.ctx),
                c(self.pts2), c(self.cos), c(self.sin))


def make_inputs(geom: ref.Geometry, grid=(8, 8, 16), s: int = 128, seed: int = 0,
                rope_layout: str = "axes", k_rows: int = 1, adaln: str = "mlp",
                x_std: float = 1.0) -> BlockInputs:
    """Block inputs for a latent grid (F, H, W): x, ctx N(0, 1);
    tstab/pts2 from the adaln MLP at t = 0.5 (adaln="mlp", K = 1) or drawn
    N(0, 0.1) with K rows and a striped tidx (adaln="random")."""
    f, h, w = grid
    t = f * h * w
    d = geom.d
    x = normal_f32(seed, "x", (t, d), x_std)
    ctx = normal_f32(seed, "ctx", (s, d), 1.0)
    if adaln == "mlp":
        tstab, pts2 = adaln_tables(d, seed)
        if k_rows > 1:
            tstab = np.concatenate([tstab] + [normal_f32(seed, f"tstab{k}", (1, 9, d), 0.1)
                                              for k in range(1, k_rows)], axis=0)
    else:
        tstab = normal_f32(seed, "tstab", (k_rows, 9, d), 0.1)
        pts2 = normal_f32(seed, "pts2", (2, d), 0.1)
    tidx = (np.arange(t) * k_rows // t).astype(np.int32) if k_rows > 1 else np.zeros(t, np.int32)
    pos = grid_positions(f, h, w)
    if rope_layout == "axes":
        cos, sin = rope_axes(pos, geom.h)
    else:
        g = np.stack([pos.T, pos.T], axis=-1).astype(np.float32)   # [3, T, 2], start == end
        cos, sin = rope_ltx(g, d, geom.h)
    return BlockInputs(x, tstab, tidx, ctx, pts2, cos, sin)
