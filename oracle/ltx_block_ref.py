"""CPU oracle for the LTX-2.5 DiT block -- TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` /
`--impl reference` legs of `bench.py` may import this module, and only as the
checker or the timed CPU baseline. The product path (the C-ABI library under
`ltx-zml_b200/`) never calls it.

What it is: a float64 (or any torch dtype) restatement of the reference's
traced block, `ltx/block.zig`, op for op:

  lin              ltx/block.zig:22-26    y = x . W^T (+ b), W upcast from bf16
  rms_no_w/rms_w   ltx/block.zig:28-34    x * rsqrt(mean(x^2) + 1e-6) (* w)
  modulate         ltx/block.zig:36-38    n * (1 + scale) + shift
  ada_val          ltx/block.zig:47-67    sst[i] + tstab[tidx[t], i] (row 0 for
                                          tidx outside [0, K): the select chain)
  rope             ltx/block.zig:71-77    split-half rotation, pairs (i, i+64)
  while_sdpa       ltx/block.zig:105-154  online softmax over K/V chunks,
                                          1/sqrt(hd) applied to K, m0 = -FLT_MAX
  sdpa_dense       zml.nn.sdpa as used at ltx/block.zig:234,525,563
  Block.attention  ltx/block.zig:212-244  qk-norm over full D, RoPE, SDPA,
                                          2*sigmoid per-head gate, out-proj
  Block stages     ltx/block.zig:248-353  s1 ... s7, block_out, w_block_out,
                                          w_attn1, f_logits; staged_rows (the
                                          stages on sampled query rows of a
                                          full-length input)
  dq / lin_q       ltx/block.zig:462-477  int8 grouped-128 dequant linear
  QBlock           ltx/block.zig:481-611  the block on dequantised weights of a
                                          field set: q_block_out_all (q/k/v x2 +
                                          FFN), qBlockOut (q/k/v x2), the probes
  quant_probes     ltx/block_conformance.zig:488-494  the five quant budgets

Parity status: the block arithmetic is **parity unpinned** against reference
artifacts. The reference is Zig on ZML/XLA (no zig/bazel here) and its own f64
oracle needs ltx_core 1.2.0 plus gated checkpoint bundles that are absent. The
restatement is pinned instead by internal known-answer tests (staged ==
one-shot, online softmax == dense, RoPE identity slots) and, for the byte-level
parts (int8 g128 quantiser, blob packing), by golden vectors produced by
running the reference's own `tools/quantize_block.py` and `tools/pack_block.py`
(see `tests/golden/make_golden.py`).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

# Reference constants, ltx/block.zig:12-18 (T/S there are harness defaults).
D = 4096
H = 32
HD = 128
FF = 16384
EPS = 1e-6
FLT_MAX = float(np.finfo(np.float32).max)

# Reference chunk sizes, ltx/block.zig:87 and :94.
ACHUNK = 16
PCHUNK = 1024


# ---------------------------------------------------------------------------
# elementwise pieces
# ---------------------------------------------------------------------------

def lin(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """ltx/block.zig:22-26: x . W^T with W (bf16 in the checkpoint) upcast."""
    y = x @ w.to(x.dtype).T
    if b is not None:
        y = y + b.to(x.dtype)
    return y


def rms_no_w(x: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    """ltx/block.zig:28-30: weightless RMSNorm over the last axis."""
    return x * torch.rsqrt((x * x).mean(dim=-1, keepdim=True) + eps)


def rms_w(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """ltx/block.zig:32-34: weighted RMSNorm (q/k norm over the full D)."""
    return rms_no_w(x) * w.to(x.dtype)


def modulate(n: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor) -> torch.Tensor:
    """ltx/block.zig:36-38."""
    return n * (scale + 1.0) + shift


def table_index(tidx: torch.Tensor, rows: int) -> torch.Tensor:
    """The table row the select chain of ltx/block.zig:58-66 picks for each
    token: tidx[t] when 0 <= tidx[t] < rows, else row 0."""
    k = tidx.long()
    return torch.where((k >= 0) & (k < rows), k, torch.zeros_like(k))


def ada_val(table: torch.Tensor, tstab: torch.Tensor, tidx: torch.Tensor, i: int) -> torch.Tensor:
    """ltx/block.zig:47-67: per-token row tstab[tidx[t], i] plus table row i.

    The reference selects rows with a select chain: row 0 everywhere, then
    row k wherever tidx == k for k = 1 .. K-1 (a bit-exact copy). An index
    gather with every tidx outside [0, K) sent to row 0 is the same selection
    (select_chain_rows below restates the chain itself for small K)."""
    chunk = tstab[:, i, :]                    # [K, D]
    tv = chunk[table_index(tidx, chunk.shape[0])]   # [T, D]
    return tv + table[i].to(tv.dtype)


def select_chain_rows(chunk: torch.Tensor, tidx: torch.Tensor) -> torch.Tensor:
    """The select chain of ltx/block.zig:58-66 as written: chunk [K, D],
    tidx [T] -> [T, D]; row 0 by default, row k where tidx == k."""
    tv = chunk[0:1].expand(tidx.shape[0], -1)
    for k in range(1, chunk.shape[0]):
        tv = torch.where((tidx == k)[:, None], chunk[k][None, :], tv)
    return tv


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """ltx/block.zig:71-77 with the [T, H, 2, 64] view of ltx/block.zig:221-226.

    x: [T, H*128]; cos/sin: [T, H, 64]. Pairs are (i, i+64) inside a head."""
    t = x.shape[0]
    h = cos.shape[1]
    x4 = x.reshape(t, h, 2, 64)
    a, b = x4[:, :, 0, :], x4[:, :, 1, :]
    c, s = cos.to(x.dtype), sin.to(x.dtype)
    ra = a * c - b * s
    rb = b * c + a * s
    return torch.cat([ra, rb], dim=-1).reshape(t, h * 128)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """GELU, tanh approximation (the FFN activation; docs/lab-notebook.md:686)."""
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)))


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------

def sdpa_dense(q3: torch.Tensor, k3: torch.Tensor, v3: torch.Tensor) -> torch.Tensor:
    """Dense softmax attention, scale applied to K (zml.nn.sdpa semantics as
    used at ltx/block.zig:234). q3 [Tq,H,hd], k3/v3 [Tk,H,hd] -> [Tq,H,hd]."""
    hd = q3.shape[-1]
    k = k3 * (1.0 / math.sqrt(hd))
    s = torch.einsum("qhd,khd->hqk", q3, k)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, v3)


def while_sdpa_c(chunk: int, q3: torch.Tensor, k3: torch.Tensor, v3: torch.Tensor) -> torch.Tensor:
    """ltx/block.zig:110-154: the loop-carried (m, l, acc) online softmax.

    m starts at -FLT_MAX (finite, so the first correction underflows to 0)."""
    tq, h, hd = q3.shape
    tk = k3.shape[0]
    assert tk % chunk == 0
    k = k3 * (1.0 / math.sqrt(hd))
    m = torch.full((h, tq), -FLT_MAX, dtype=q3.dtype)
    l = torch.zeros((h, tq), dtype=q3.dtype)
    acc = torch.zeros((h, tq, hd), dtype=q3.dtype)
    for off in range(0, tk, chunk):
        kc = k[off:off + chunk]
        vc = v3[off:off + chunk]
        s = torch.einsum("qhd,khd->hqk", q3, kc)
        cmax = s.amax(dim=-1)
        m_new = torch.maximum(m, cmax)
        corr = torch.exp(m - m_new)
        p = s.sub_(m_new[..., None]).exp_()   # exp(s - m_new), in the score buffer
        l = l * corr + p.sum(dim=-1)
        acc = acc * corr[..., None] + torch.einsum("hqk,khd->hqd", p, vc)
        m = m_new
    return (acc / l[..., None]).permute(1, 0, 2)


def while_sdpa(q3, k3, v3):
    """ltx/block.zig:105-108: chunk 1024 when it divides T_kv, else 16."""
    if k3.shape[0] % PCHUNK == 0:
        return while_sdpa_c(PCHUNK, q3, k3, v3)
    return while_sdpa_c(ACHUNK, q3, k3, v3)


# ---------------------------------------------------------------------------
# weights
# ---------------------------------------------------------------------------

# ltx/block.zig:377-406 (field -> reference file stem, dims in units of D/H/FF)
WEIGHT_SPECS = [
    ("q1_w", "attn1_to_q_weight", ("D", "D")), ("q1_b", "attn1_to_q_bias", ("D",)),
    ("k1_w", "attn1_to_k_weight", ("D", "D")), ("k1_b", "attn1_to_k_bias", ("D",)),
    ("v1_w", "attn1_to_v_weight", ("D", "D")), ("v1_b", "attn1_to_v_bias", ("D",)),
    ("o1_w", "attn1_to_out_0_weight", ("D", "D")), ("o1_b", "attn1_to_out_0_bias", ("D",)),
    ("qn1", "attn1_q_norm_weight", ("D",)), ("kn1", "attn1_k_norm_weight", ("D",)),
    ("g1_w", "attn1_to_gate_logits_weight", ("H", "D")), ("g1_b", "attn1_to_gate_logits_bias", ("H",)),
    ("q2_w", "attn2_to_q_weight", ("D", "D")), ("q2_b", "attn2_to_q_bias", ("D",)),
    ("k2_w", "attn2_to_k_weight", ("D", "D")), ("k2_b", "attn2_to_k_bias", ("D",)),
    ("v2_w", "attn2_to_v_weight", ("D", "D")), ("v2_b", "attn2_to_v_bias", ("D",)),
    ("o2_w", "attn2_to_out_0_weight", ("D", "D")), ("o2_b", "attn2_to_out_0_bias", ("D",)),
    ("qn2", "attn2_q_norm_weight", ("D",)), ("kn2", "attn2_k_norm_weight", ("D",)),
    ("g2_w", "attn2_to_gate_logits_weight", ("H", "D")), ("g2_b", "attn2_to_gate_logits_bias", ("H",)),
    ("ff1_w", "ff_net_0_proj_weight", ("FF", "D")),
    ("ff2_w", "ff_net_2_weight", ("D", "FF")),
    ("sst", "scale_shift_table", (9, "D")),
    ("psst", "prompt_scale_shift_table", (2, "D")),
]
F32_FIELDS = ("sst", "psst")

# ltx/loader.zig:147-156: the int8 set of the reference's quantised block.
Q8_FIELDS = ("q1_w", "k1_w", "v1_w", "q2_w", "k2_w", "v2_w", "ff1_w", "ff2_w")
# BASELINE's extension: output projections quantised too.
Q8_FIELDS_EXT = Q8_FIELDS + ("o1_w", "o2_w")
# QBlock.qBlockOut's set (ltx/block.zig:577-611): q/k/v of both attentions,
# the FFN left unquantised.
Q8_FIELDS_QKV = ("q1_w", "k1_w", "v1_w", "q2_w", "k2_w", "v2_w")


@dataclass
class Geometry:
    d: int = D
    ff: int = FF

    @property
    def h(self) -> int:
        return self.d // HD

    def dims(self, spec):
        m = {"D": self.d, "H": self.h, "FF": self.ff}
        return tuple(m.get(s, s) if isinstance(s, str) else s for s in spec)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round f32 values to bf16 (round-to-nearest-even), returned as uint16."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    return r


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# int8 grouped-128 quantiser -- tools/quantize_block.py:52-59 (+ bf16 scales)
# ---------------------------------------------------------------------------

def quantize_g128(w: np.ndarray, gs: int = 128, bits: int = 8, scale_dtype: str = "f32"):
    """Symmetric grouped absmax quantiser, tools/quantize_block.py:40-59.

    q = clip(round(w / s), lo, qmax), s = absmax / qmax per [row, group]
    (s = 1 where absmax == 0), computed in float64 from the f32 weights.
    Returns (q int8 [O, I], scale [O, I/gs] as float32 or bf16-as-uint16).

    scale_dtype "bf16" (the BASELINE configs) rounds the f64 scale to bf16
    *before* quantising, so q is consistent with the scale the kernel uses."""
    qmax = 7 if bits == 4 else 127
    lo = -8 if bits == 4 else -128
    w = np.asarray(w, dtype=np.float64)
    o, i = w.shape
    wg = w.reshape(o, i // gs, gs)
    absmax = np.abs(wg).max(axis=2, keepdims=True)
    scale3 = np.where(absmax > 0, absmax / qmax, 1.0)
    if scale_dtype == "bf16":
        s16 = bf16_round(scale3.astype(np.float32))
        scale3 = bf16_to_f32(s16).astype(np.float64)
    q = np.clip(np.round(wg / scale3), lo, qmax).astype(np.int8).reshape(o, i)
    if scale_dtype == "bf16":
        return q, s16.reshape(o, i // gs)
    return q, scale3.squeeze(2).astype(np.float32)


def dequant(q: np.ndarray, scale: np.ndarray, gs: int = 128) -> np.ndarray:
    """ltx/block.zig:462-471 (dq4 on i8): w[o, g, e] = q[o, g, e] * sc[o, g],
    in float64 (exact for int8 x f32/bf16 scales)."""
    if scale.dtype == np.uint16:
        scale = bf16_to_f32(scale)
    o, i = q.shape
    f = q.astype(np.float64).reshape(o, i // gs, gs) * scale.astype(np.float64)[:, :, None]
    return f.reshape(o, i)


# ---------------------------------------------------------------------------
# the block
# ---------------------------------------------------------------------------

@dataclass
class BlockWeights:
    """One block's weights as torch tensors (float dtype of the oracle run).

    `raw` keeps the stored form (bf16 bits as uint16, f32, or int8 + scale)
    so the same bytes can be uploaded to the GPU library."""
    t: dict = field(default_factory=dict)
    raw: dict = field(default_factory=dict)
    geom: Geometry = field(default_factory=Geometry)


class Block:
    """ltx/block.zig:156-366 restated. All tensors are 2-D [tokens, D]."""

    def __init__(self, w: BlockWeights, dtype=torch.float64):
        self.w = {k: v.to(dtype) for k, v in w.t.items()}
        self.h = w.geom.h
        self.dtype = dtype

    def attention(self, idx, x, ctx, pe, gated, algo):
        """ltx/block.zig:212-244 (idx 1 = self-attention, 2 = cross)."""
        def lin_(a, wname, bname):
            return lin(a, self.w[wname], self.w[bname])
        n = str(idx)
        tq, tk = x.shape[0], ctx.shape[0]
        q = rms_w(lin_(x, f"q{n}_w", f"q{n}_b"), self.w[f"qn{n}"])
        k = rms_w(lin_(ctx, f"k{n}_w", f"k{n}_b"), self.w[f"kn{n}"])
        v = lin_(ctx, f"v{n}_w", f"v{n}_b")
        if pe is not None:
            cos, sin = pe
            q = rope(q, cos, sin)
            k = rope(k, cos, sin)
        q3 = q.reshape(tq, self.h, HD)
        k3 = k.reshape(tk, self.h, HD)
        v3 = v.reshape(tk, self.h, HD)
        out = sdpa_dense(q3, k3, v3) if algo == "dense" else while_sdpa(q3, k3, v3)
        if gated:
            glog = lin(x, self.w[f"g{n}_w"], self.w[f"g{n}_b"])       # [T, H]
            gate = torch.sigmoid(glog) * 2.0
            out = out * gate[:, :, None]
        merged = out.reshape(tq, self.h * HD)
        return lin_(merged, f"o{n}_w", f"o{n}_b")

    # ---- stages (ltx/block.zig:248-353) ----
    def s1_norm_msa(self, x, tstab, tidx):
        shift = ada_val(self.w["sst"], tstab, tidx, 0)
        scl = ada_val(self.w["sst"], tstab, tidx, 1)
        return modulate(rms_no_w(x), scl, shift)

    def s1b_qnorm(self, x, tstab, tidx):
        n = self.s1_norm_msa(x, tstab, tidx)
        return rms_w(lin(n, self.w["q1_w"], self.w["q1_b"]), self.w["qn1"])

    def s2_attn1_nogate(self, x, tstab, tidx, cos, sin):
        n = self.s1_norm_msa(x, tstab, tidx)
        return self.attention(1, n, n, (cos, sin), False, "dense")

    def attn1_out(self, x, tstab, tidx, cos, sin, algo="dense"):
        n = self.s1_norm_msa(x, tstab, tidx)
        return self.attention(1, n, n, (cos, sin), True, algo)

    def s3_attn1(self, x, tstab, tidx, cos, sin):
        return self.attn1_out(x, tstab, tidx, cos, sin, "dense")

    def w_attn1(self, x, tstab, tidx, cos, sin):
        """ltx/block.zig:274-276: attn1 with the blockwise online softmax."""
        return self.attn1_out(x, tstab, tidx, cos, sin, "blockwise")

    def f_logits(self, x, tstab, tidx, cos, sin):
        """ltx/block.zig:356-365: self-attention's pre-softmax logits q.k over
        hd (no 1/sqrt(hd) scale), after q/k norm and RoPE -> [Tq, H, Tk]."""
        n = self.s1_norm_msa(x, tstab, tidx)
        q = rope(rms_w(lin(n, self.w["q1_w"], self.w["q1_b"]), self.w["qn1"]), cos, sin)
        k = rope(rms_w(lin(n, self.w["k1_w"], self.w["k1_b"]), self.w["kn1"]), cos, sin)
        t = q.shape[0]
        return torch.einsum("qhd,khd->qhk", q.reshape(t, self.h, HD), k.reshape(t, self.h, HD))

    def after_sa(self, x, tstab, tidx, cos, sin, algo="dense"):
        gate = ada_val(self.w["sst"], tstab, tidx, 2)
        return x + self.attn1_out(x, tstab, tidx, cos, sin, algo) * gate

    def s4_after_sa(self, x, tstab, tidx, cos, sin):
        return self.after_sa(x, tstab, tidx, cos, sin)

    def s4_normed(self, x, tstab, tidx, cos, sin):
        return rms_no_w(self.after_sa(x, tstab, tidx, cos, sin))

    def ca_out(self, x_normed, tstab, tidx, ctx, pts2):
        """ltx/block.zig:291-306."""
        shift_q = ada_val(self.w["sst"], tstab, tidx, 6)
        scale_q = ada_val(self.w["sst"], tstab, tidx, 7)
        gate_ca = ada_val(self.w["sst"], tstab, tidx, 8)
        attn_in = modulate(x_normed, scale_q, shift_q)
        kv = self.w["psst"] + pts2.to(self.dtype)
        enc = ctx * (kv[1] + 1.0) + kv[0]
        ca = self.attention(2, attn_in, enc, None, True, "dense")
        return ca * gate_ca

    def s5_ca_out(self, x, tstab, tidx, ctx, pts2, cos, sin, algo="dense"):
        return self.ca_out(rms_no_w(self.after_sa(x, tstab, tidx, cos, sin, algo)), tstab, tidx, ctx, pts2)

    def s6_ff_in(self, x, tstab, tidx, ctx, pts2, cos, sin):
        x_sa = self.after_sa(x, tstab, tidx, cos, sin)
        x_ca = x_sa + self.ca_out(rms_no_w(x_sa), tstab, tidx, ctx, pts2)
        return modulate(rms_no_w(x_ca), ada_val(self.w["sst"], tstab, tidx, 4),
                        ada_val(self.w["sst"], tstab, tidx, 3))

    def ffn(self, ff_in):
        return lin(gelu_tanh(lin(ff_in, self.w["ff1_w"])), self.w["ff2_w"])

    def s7_ff_out(self, x, tstab, tidx, ctx, pts2, cos, sin):
        return self.ffn(self.s6_ff_in(x, tstab, tidx, ctx, pts2, cos, sin))

    def block_out_a(self, x, tstab, tidx, ctx, pts2, cos, sin, algo="dense"):
        """ltx/block.zig:340-344, computed once (no prefix recompute)."""
        x_sa = self.after_sa(x, tstab, tidx, cos, sin, algo)
        x_ca = x_sa + self.ca_out(rms_no_w(x_sa), tstab, tidx, ctx, pts2)
        ff_in = modulate(rms_no_w(x_ca), ada_val(self.w["sst"], tstab, tidx, 4),
                         ada_val(self.w["sst"], tstab, tidx, 3))
        return x_ca + self.ffn(ff_in) * ada_val(self.w["sst"], tstab, tidx, 5)

    def block_out(self, *a):
        return self.block_out_a(*a, algo="dense")

    def w_block_out(self, *a):
        return self.block_out_a(*a, algo="blockwise")

    def staged(self, x, tstab, tidx, ctx, pts2, cos, sin):
        """All ten conformance stages of ltx/block_conformance.zig:311-322,
        computed in one pass (each equals the reference's prefix-recomputing
        stage method)."""
        out = {}
        n = self.s1_norm_msa(x, tstab, tidx)
        out["s1_norm_msa"] = n
        out["s1b_qnorm"] = rms_w(lin(n, self.w["q1_w"], self.w["q1_b"]), self.w["qn1"])
        out["s2_attn1_nogate"] = self.attention(1, n, n, (cos, sin), False, "dense")
        a1 = self.attention(1, n, n, (cos, sin), True, "dense")
        out["s3_attn1"] = a1
        x_sa = x + a1 * ada_val(self.w["sst"], tstab, tidx, 2)
        out["s4_after_sa"] = x_sa
        xn = rms_no_w(x_sa)
        out["s4_normed"] = xn
        ca = self.ca_out(xn, tstab, tidx, ctx, pts2)
        out["s5_ca_out"] = ca
        x_ca = x_sa + ca
        ff_in = modulate(rms_no_w(x_ca), ada_val(self.w["sst"], tstab, tidx, 4),
                         ada_val(self.w["sst"], tstab, tidx, 3))
        out["s6_ff_in"] = ff_in
        ff = self.ffn(ff_in)
        out["s7_ff_out"] = ff
        out["block_out"] = x_ca + ff * ada_val(self.w["sst"], tstab, tidx, 5)
        return out


    def staged_rows(self, x, tstab, tidx, ctx, pts2, cos, sin, rows, head_group: int = 8):
        """`staged` for the query rows `rows` only (a full-length run checked
        on sampled rows). Every stage of ltx/block.zig:248-353 is per token
        except self-attention, whose keys and values come from all T tokens:
        K = rope(rmsW(lin(n, k1)), cos, sin) and V = lin(n, v1) are computed
        over every row (ltx/block.zig:212-231), the queries only for `rows`
        with those rows' cos/sin. Dense softmax over all T keys, `head_group`
        heads at a time to bound the score buffer. Returns
        {stage: [len(rows), D]}."""
        w = self.w
        rows = torch.as_tensor(np.asarray(rows), dtype=torch.long)
        n_all = self.s1_norm_msa(x, tstab, tidx)
        k_all = rope(rms_w(lin(n_all, w["k1_w"], w["k1_b"]), w["kn1"]), cos, sin)
        v_all = lin(n_all, w["v1_w"], w["v1_b"])
        n = n_all[rows]
        del n_all
        xr, tr = x[rows], tidx[rows]
        out = {"s1_norm_msa": n}
        qn = rms_w(lin(n, w["q1_w"], w["q1_b"]), w["qn1"])
        out["s1b_qnorm"] = qn
        q = rope(qn, cos[rows], sin[rows])
        r, t = q.shape[0], k_all.shape[0]
        q3 = q.reshape(r, self.h, HD)
        k3 = k_all.reshape(t, self.h, HD)
        v3 = v_all.reshape(t, self.h, HD)
        att = torch.cat([sdpa_dense(q3[:, h0:h0 + head_group], k3[:, h0:h0 + head_group],
                                    v3[:, h0:h0 + head_group]) for h0 in range(0, self.h, head_group)], dim=1)
        del k_all, v_all, k3, v3
        out["s2_attn1_nogate"] = lin(att.reshape(r, self.h * HD), w["o1_w"], w["o1_b"])
        gate = torch.sigmoid(lin(n, w["g1_w"], w["g1_b"])) * 2.0           # ltx/block.zig:236-240
        a1 = lin((att * gate[:, :, None]).reshape(r, self.h * HD), w["o1_w"], w["o1_b"])
        out["s3_attn1"] = a1
        x_sa = xr + a1 * ada_val(w["sst"], tstab, tr, 2)
        out["s4_after_sa"] = x_sa
        xn = rms_no_w(x_sa)
        out["s4_normed"] = xn
        ca = self.ca_out(xn, tstab, tr, ctx, pts2)
        out["s5_ca_out"] = ca
        x_ca = x_sa + ca
        ff_in = modulate(rms_no_w(x_ca), ada_val(w["sst"], tstab, tr, 4), ada_val(w["sst"], tstab, tr, 3))
        out["s6_ff_in"] = ff_in
        ff = self.ffn(ff_in)
        out["s7_ff_out"] = ff
        out["block_out"] = x_ca + ff * ada_val(w["sst"], tstab, tr, 5)
        return out


STAGES = ["s1_norm_msa", "s1b_qnorm", "s2_attn1_nogate", "s3_attn1", "s4_after_sa",
          "s4_normed", "s5_ca_out", "s6_ff_in", "s7_ff_out", "block_out"]


class QBlock(Block):
    """ltx/block.zig:481-574: the Block with int8 g128 linears.

    `qset` lists which weight fields are replaced by their dequantised form;
    the reference's qBlockOutAll quantises Q8_FIELDS (ltx/loader.zig:147-156).
    Dequantisation is exact in float64, so this is Block on dequantised
    weights -- which is what ltx/block.zig:473-477 computes."""

    def __init__(self, w: BlockWeights, dtype=torch.float64, qset=Q8_FIELDS):
        super().__init__(w, dtype)
        for f in qset:
            q, sc = w.raw[f + "::q8"], w.raw[f + "::q8scale"]
            self.w[f] = torch.from_numpy(dequant(q, sc)).to(dtype)

    def q_block_out_all(self, *a):
        return self.block_out(*a)


# The reference's quantisation probes (ltx/block_conformance.zig:488-494):
# (Block method, QBlock method, the weights QBlock's method quantises, budget
# of rel-RMS(q, f)). QBlock's probe methods quantise only the linears they
# name (ltx/block.zig:513-611): qLogits q1/k1 (:513-517), qAttn1 q1/k1/v1
# (:520-530), qBlockOut q/k/v of both attentions (:577-611), qFfOut the FFN
# applied to the unquantised block's s6FfIn (:539-541), qBlockOutAll the
# reference int8 set (:544-574). With QBlock = the block on dequantised
# weights, each probe is the Block method on that field set.
QUANT_PROBES = [
    ("f_logits", ("q1_w", "k1_w"), 5e-2),
    ("s3_attn1", ("q1_w", "k1_w", "v1_w"), 2e-2),
    ("block_out", Q8_FIELDS_QKV, 2e-2),
    ("s7_ff_out", ("ff1_w", "ff2_w"), 5e-2),
    ("block_out", Q8_FIELDS, 2e-2),
]
PROBE_NAMES = {"f_logits": ("fLogits", "qLogits"), "s3_attn1": ("s3Attn1", "qAttn1"),
               "s7_ff_out": ("s7FfOut", "qFfOut")}


def quant_probes(w: BlockWeights, x, tstab, tidx, ctx, pts2, cos, sin, dtype=torch.float64) -> list:
    """The probe table above on one input: [(f name, q name, rel-RMS, budget)]."""
    base = Block(w, dtype)
    out = []
    for meth, fields, budget in QUANT_PROBES:
        qb = QBlock(w, dtype, qset=fields)
        if meth in ("f_logits", "s3_attn1"):
            args = (x, tstab, tidx, cos, sin)
        else:
            args = (x, tstab, tidx, ctx, pts2, cos, sin)
        f = getattr(base, meth)(*args)
        q = getattr(qb, meth)(*args)
        fn, qn = PROBE_NAMES.get(meth, ("blockOut", "qBlockOutAll" if fields == Q8_FIELDS else "qBlockOut"))
        out.append((fn, qn, rel_rms(q, f), budget))
    return out


def rel_rms(got, want) -> float:
    """ltx/block_conformance.zig:183-215: sqrt(sum (g-w)^2 / (sum w^2 + 1e-20))."""
    g = np.asarray(got, dtype=np.float64).ravel()
    w = np.asarray(want, dtype=np.float64).ravel()
    return float(np.sqrt(((g - w) ** 2).sum() / ((w * w).sum() + 1e-20)))


def max_abs(got, want) -> float:
    g = np.asarray(got, dtype=np.float64).ravel()
    w = np.asarray(want, dtype=np.float64).ravel()
    return float(np.abs(g - w).max()) if g.size else 0.0
