"""Core parts and scheduler of the denoising step -- TEST INFRASTRUCTURE ONLY.

CPU restatement (the checker for the GPU library's device-side core parts
and scheduler; nothing here ships or is timed as the product):

* core parts, ltx/core_parts.zig:21-181: the f32 sinusoid of t*1000 (cos
  half first, divisor 128), embedded_timestep = linear_2(SiLU(linear_1(.))),
  ts9 = adaln linear(SiLU(emb)) in the block's [K, 9, D] table layout, pts2
  from the prompt adaln MLP in [2, D], patchify (128 -> D, bias), and the
  output tail: mean-subtracting LayerNorm (biased variance, eps 1e-6), then
  x*(1+scale)+shift with shift/scale = scale_shift_table rows 0/1 + the RAW
  embedded_timestep, then proj_out (D -> 128, bias). Arithmetic in f64 after
  the f32 sinusoid (the reference's oracle convention, bf16 weights
  upcast).
* scheduler, ltx/scheduler.zig:11-80: the distilled sigma lists; torch.lerp's
  two-branch fused form; noise init; timesteps = mask * sigma;
  to_denoised, post_process and the Euler step in f32 with no fused
  multiply-add (bit-exact targets).

Checkpoint names of the core tensors follow ltx/core_parts.zig:52-70.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import inputs as oin
from . import ltx_block_ref as ref

IN_CH = 128
EPS = 1e-6

# field -> (checkpoint stem without extension, shape factory, dtype)
CORE_SPECS = {
    "ada_l1_w": ("adaln_single.emb.timestep_embedder.linear_1.weight", lambda d: (d, 256), "bf16"),
    "ada_l1_b": ("adaln_single.emb.timestep_embedder.linear_1.bias", lambda d: (d,), "bf16"),
    "ada_l2_w": ("adaln_single.emb.timestep_embedder.linear_2.weight", lambda d: (d, d), "bf16"),
    "ada_l2_b": ("adaln_single.emb.timestep_embedder.linear_2.bias", lambda d: (d,), "bf16"),
    "ada_out_w": ("adaln_single.linear.weight", lambda d: (9 * d, d), "bf16"),
    "ada_out_b": ("adaln_single.linear.bias", lambda d: (9 * d,), "bf16"),
    "pada_l1_w": ("prompt_adaln_single.emb.timestep_embedder.linear_1.weight", lambda d: (d, 256), "bf16"),
    "pada_l1_b": ("prompt_adaln_single.emb.timestep_embedder.linear_1.bias", lambda d: (d,), "bf16"),
    "pada_l2_w": ("prompt_adaln_single.emb.timestep_embedder.linear_2.weight", lambda d: (d, d), "bf16"),
    "pada_l2_b": ("prompt_adaln_single.emb.timestep_embedder.linear_2.bias", lambda d: (d,), "bf16"),
    "pada_out_w": ("prompt_adaln_single.linear.weight", lambda d: (2 * d, d), "bf16"),
    "pada_out_b": ("prompt_adaln_single.linear.bias", lambda d: (2 * d,), "bf16"),
    "pat_w": ("patchify_proj.weight", lambda d: (d, IN_CH), "bf16"),
    "pat_b": ("patchify_proj.bias", lambda d: (d,), "bf16"),
    "po_w": ("proj_out.weight", lambda d: (IN_CH, d), "bf16"),
    "po_b": ("proj_out.bias", lambda d: (IN_CH,), "bf16"),
    "fsst": ("scale_shift_table", lambda d: (2, d), "f32"),
}


@dataclass
class CoreWeights:
    d: int
    raw: dict = field(default_factory=dict)  # field -> uint16 bf16 bits or f32 array (what is stored)
    t: dict = field(default_factory=dict)    # field -> float64 torch tensor (exact values)


def make_core_weights(d: int, seed: int = 0, std: float = 0.02) -> CoreWeights:
    """N(0, std) weights and biases materialised as bf16, scale_shift_table
    N(0, std) f32 (the checkpoint's lone f32 video tensor)."""
    cw = CoreWeights(d)
    for f, (_, shape, dt) in CORE_SPECS.items():
        a = oin.normal_f32(seed, "core_" + f, shape(d), std)
        if dt == "bf16":
            u, t = oin.bf16_tensor(a)
            cw.raw[f], cw.t[f] = u, t
        else:
            cw.raw[f], cw.t[f] = a, torch.from_numpy(a.astype(np.float64))
    return cw


def core_tensors(cw: CoreWeights):
    """(name, dtype, shape, bytes) of the core tensors for oracle.blob.pack."""
    out = []
    for f, (name, shape, dt) in CORE_SPECS.items():
        a = cw.raw[f]
        out.append((name, "F32" if dt == "f32" else "BF16", list(shape(cw.d)), a.tobytes()))
    return out


def _silu(x: torch.Tensor) -> torch.Tensor:
    return x * torch.sigmoid(x)


def layer_norm_no_w(x: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    """ltx/core_parts.zig:30-35: mean-subtracting, biased variance."""
    c = x - x.mean(-1, keepdim=True)
    return c * torch.rsqrt((c * c).mean(-1, keepdim=True) + eps)


class CoreParts:
    def __init__(self, cw: CoreWeights):
        self.w = cw.t
        self.d = cw.d

    def emb(self, t: np.ndarray) -> torch.Tensor:
        """embedded_timestep [K, D] (ltx/core_parts.zig:117-119)."""
        s = torch.from_numpy(oin.sinusoid_f32(np.asarray(t, dtype=np.float32)).astype(np.float64))
        w = self.w
        return ref.lin(_silu(ref.lin(s, w["ada_l1_w"], w["ada_l1_b"])), w["ada_l2_w"], w["ada_l2_b"])

    def ts9r(self, t: np.ndarray) -> torch.Tensor:
        """[K, 9, D] (ltx/core_parts.zig:122-124, :135-137)."""
        w = self.w
        return ref.lin(_silu(self.emb(t)), w["ada_out_w"], w["ada_out_b"]).reshape(-1, 9, self.d)

    def pts2r(self, sigma: float) -> torch.Tensor:
        """[2, D] (ltx/core_parts.zig:127-131, :140-142)."""
        w = self.w
        s = torch.from_numpy(oin.sinusoid_f32(np.asarray([sigma], dtype=np.float32)).astype(np.float64))
        e = ref.lin(_silu(ref.lin(s, w["pada_l1_w"], w["pada_l1_b"])), w["pada_l2_w"], w["pada_l2_b"])
        return ref.lin(_silu(e), w["pada_out_w"], w["pada_out_b"]).reshape(2, self.d)

    def patchify(self, latent: torch.Tensor) -> torch.Tensor:
        """[T, 128] -> [T, D] (ltx/core_parts.zig:144-146)."""
        return ref.lin(latent, self.w["pat_w"], self.w["pat_b"])

    def tail_from_emb(self, x: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
        """x [T, D], e [T, D] (embedded_timestep per token) -> velocity [T, 128]
        (ltx/core_parts.zig:148-170)."""
        shift = self.w["fsst"][0][None, :] + e
        scale = self.w["fsst"][1][None, :] + e
        return ref.lin(ref.modulate(layer_norm_no_w(x), scale, shift), self.w["po_w"], self.w["po_b"])


# ---------------------------------------------------------------------------
# scheduler (bit-exact f32)
# ---------------------------------------------------------------------------

SIGMAS_STAGE1 = np.array([1.0, 0.99375, 0.9875, 0.98125, 0.975, 0.909375, 0.725, 0.421875, 0.0], dtype=np.float32)
SIGMAS_STAGE2 = np.array([0.909375, 0.725, 0.421875, 0.0], dtype=np.float32)


def fma32(a, b, c) -> np.ndarray:
    """Correctly rounded f32 a*b + c (one rounding). The product is exact in
    f64 and the f64 sum's error e is recovered exactly (TwoSum). Rounding the
    f64 sum s to f32 can differ from rounding the exact value s + e only when
    s lies exactly halfway between two f32 neighbours; then the sign of e
    picks the neighbour."""
    a, b, c = (np.asarray(v, dtype=np.float32) for v in (a, b, c))
    a, b, c = np.broadcast_arrays(a, b, c)
    p = a.astype(np.float64) * b.astype(np.float64)
    c64 = c.astype(np.float64)
    s = p + c64
    bp = s - p
    e = (p - (s - bp)) + (c64 - bp)
    r = s.astype(np.float32)
    up = np.nextafter(r, np.float32(np.inf))
    dn = np.nextafter(r, np.float32(-np.inf))
    r64 = r.astype(np.float64)
    mid_hi = s == (r64 + up.astype(np.float64)) / 2   # s halfway between r and up
    mid_lo = s == (r64 + dn.astype(np.float64)) / 2   # s halfway between dn and r
    out = np.where(mid_hi & (e > 0), up, r)
    out = np.where(mid_lo & (e < 0), dn, out)
    return out.astype(np.float32)


def lerp(a, b, w) -> np.ndarray:
    """torch.lerp's two-branch fused kernel (ltx/scheduler.zig:20-35)."""
    a, b, w = (np.asarray(v, dtype=np.float32) for v in (a, b, w))
    d = (b - a).astype(np.float32)
    lo = fma32(w, d, a)
    hi = fma32(-d, (np.float32(1.0) - w).astype(np.float32), b)
    return np.where(np.abs(w) < 0.5, lo, hi).astype(np.float32)


def noise_init(clean, noise, mask, noise_scale: float) -> np.ndarray:
    """ltx/scheduler.zig:37-46: x = lerp(clean, noise, scale); lerp(clean, x, mask)."""
    x = lerp(clean, noise, np.float32(noise_scale))
    return lerp(clean, x, np.asarray(mask, dtype=np.float32)[:, None])


def timesteps(mask, sigma: float) -> np.ndarray:
    return (np.asarray(mask, dtype=np.float32) * np.float32(sigma)).astype(np.float32)


def to_denoised(x, v, ts) -> np.ndarray:
    return (x - (v * np.asarray(ts, dtype=np.float32)[:, None]).astype(np.float32)).astype(np.float32)


def post_process(den, clean, mask) -> np.ndarray:
    m = np.asarray(mask, dtype=np.float32)[:, None]
    return ((den * m).astype(np.float32) + (clean * (np.float32(1.0) - m)).astype(np.float32)).astype(np.float32)


def euler_step(x, post, sigma: float, sigma_next: float) -> np.ndarray:
    dt = np.float32(np.float32(sigma_next) - np.float32(sigma))
    v = ((x - post).astype(np.float32) / np.float32(sigma)).astype(np.float32)
    return (x + (v * dt).astype(np.float32)).astype(np.float32)


def scheduler_step(x, vel, ts, clean, mask, sigma: float, sigma_next: float) -> np.ndarray:
    """The host march of ltx/e2e_denoise.zig:320-325 in one function."""
    den = to_denoised(x, vel, ts)
    post = post_process(den, clean, mask)
    return euler_step(x, post, sigma, sigma_next)


def denoise_ref(core: CoreParts, blocks: list, sigmas, latent, clean, mask, mask_values, tidx, ctx, cos, sin,
                dtype=torch.float64) -> list:
    """The loop of ltx/e2e_denoise.zig:218-336: per step, conditioning from
    the f32 timesteps, patchify, every block, the tail, then the f32 host
    march. Core parts and blocks in `dtype`; returns the latent after each
    step (f32)."""
    out = []
    lat = np.asarray(latent, dtype=np.float32)
    c = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dtype)
    tid = torch.from_numpy(np.asarray(tidx, dtype=np.int32))
    for s in range(len(sigmas) - 1):
        sg, sn = float(sigmas[s]), float(sigmas[s + 1])
        ts = timesteps(mask, sg)
        tk = timesteps(mask_values, sg)
        emb = core.emb(tk).to(dtype)
        ts9 = core.ts9r(tk).to(dtype)
        pts2 = core.pts2r(sg).to(dtype)
        x = core.patchify(c(lat)).to(dtype)
        for b in blocks:
            x = b.block_out(x, ts9, tid, c(ctx), pts2, c(cos), c(sin))
        vel = core.tail_from_emb(x.double(), emb.double()[ref.table_index(tid, emb.shape[0])]).numpy().astype(np.float32)
        lat = scheduler_step(lat, vel, ts, clean, mask, sg, sn)
        out.append(lat)
    return out
