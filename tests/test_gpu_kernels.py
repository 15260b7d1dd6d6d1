"""GPU parity tests of the standalone operators through the C ABI:
tcgen05 GEMM (bf16 and int8 grouped-128 weights, fused and unfused dequant)
and tcgen05 flash attention, against float64 CPU references of the same
inputs (BASELINE configs 1 and 2)."""

import math

import numpy as np
import pytest
import torch

from oracle import inputs as oin
from oracle import ltx_block_ref as ref

pytestmark = pytest.mark.gpu

# bf16 outputs carry a 2^-9 relative rounding; accumulation is f32.
GEMM_TOL = 4e-3
ATTN_TOL = 5e-3


def _bf16(a: np.ndarray, device):
    return torch.from_numpy(ref.bf16_to_f32(ref.bf16_round(a))).to(device).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 256), (1, 32, 128), (257, 128, 4096),
                                   (64, 768, 1024), (1000, 4096, 512)])
def test_gemm_bf16(cuda, M, N, K):
    import ltxb
    g = torch.Generator().manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, generator=g).to(cuda).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(cuda).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.02).to(cuda).to(torch.bfloat16)
    out = ltxb.gemm_bf16(a, w, b)
    torch.cuda.synchronize()
    want = a.double().cpu() @ w.double().cpu().T + b.double().cpu()
    assert ref.rel_rms(out.float().cpu(), want) < GEMM_TOL
    assert ltxb.device_status() == ltxb.OK


@pytest.mark.parametrize("scale_dtype", ["f32", "bf16"])
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (333, 384, 512), (128, 1024, 4096)])
def test_dq_gemm(cuda, scale_dtype, M, N, K):
    """linQ (ltx/block.zig:473-477): bf16 A . dequant(int8, g128 scale)^T, both
    dequant placements, against f64 on the exactly-dequantised weights."""
    import ltxb
    w = oin.apply_outliers(oin.normal_f32(M, "dq", (N, K), 0.02), M, "dq")
    q, sc = ref.quantize_g128(w, scale_dtype=scale_dtype)
    a_np = oin.normal_f32(M, "a", (M, K), 1.0)
    a = _bf16(a_np, cuda)
    b = _bf16(oin.normal_f32(M, "b", (N,), 0.02), cuda)
    wq = torch.from_numpy(q).to(cuda)
    if scale_dtype == "bf16":
        s = torch.from_numpy(sc.view(np.int16)).to(cuda).view(torch.bfloat16)
    else:
        s = torch.from_numpy(sc).to(cuda)
    fused = ltxb.dq_gemm(a, wq, s, b, fused=True)
    unfused = ltxb.dq_gemm(a, wq, s, b, fused=False)
    torch.cuda.synchronize()
    deq = ref.dequant(q, sc)
    want = a.double().cpu().numpy() @ deq.T + b.double().cpu().numpy()
    assert ref.rel_rms(fused.float().cpu(), want) < GEMM_TOL
    # same bf16 operands into the same MMA sequence: identical bits
    assert torch.equal(fused, unfused)


def test_gemm_rejects_bad_shapes(cuda):
    import ltxb
    a = torch.zeros(16, 100, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(32, 100, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(ltxb.LtxbError) as ei:
        ltxb.gemm_bf16(a, w)
    assert ei.value.code == ltxb.EINVAL
    a = torch.zeros(16, 128, device=cuda, dtype=torch.bfloat16)
    w = torch.zeros(40, 128, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(ltxb.LtxbError):
        ltxb.gemm_bf16(a, w)


def _attn_ref(q, k, v, gate=None):
    o = ref.sdpa_dense(q.double().cpu(), k.double().cpu(), v.double().cpu())
    if gate is not None:
        o = o * gate.double().cpu()[:, :, None]
    return o


@pytest.mark.parametrize("Tq,Tkv,H", [(128, 128, 1), (256, 384, 2), (200, 300, 2), (77, 128, 3), (130, 1, 1),
                                      (512, 1000, 2)])
def test_attention(cuda, Tq, Tkv, H):
    import ltxb
    g = torch.Generator().manual_seed(Tq + Tkv)
    q = torch.randn(Tq, H, 128, generator=g).to(cuda).to(torch.bfloat16)
    k = torch.randn(Tkv, H, 128, generator=g).to(cuda).to(torch.bfloat16)
    v = torch.randn(Tkv, H, 128, generator=g).to(cuda).to(torch.bfloat16)
    gate = (2 * torch.sigmoid(torch.randn(Tq, H, generator=g))).to(cuda)
    out = ltxb.attention(q, k, v, gate)
    torch.cuda.synchronize()
    assert ref.rel_rms(out.float().cpu(), _attn_ref(q, k, v, gate)) < ATTN_TOL
    assert ltxb.device_status() == ltxb.OK


def test_attention_peaked_scores(cuda):
    """Large logits force the running max to move across K/V tiles (the O
    rescale path), including a late jump in the last tile."""
    import ltxb
    g = torch.Generator().manual_seed(5)
    T, H = 384, 2
    q = torch.randn(T, H, 128, generator=g) * 3
    k = torch.randn(T, H, 128, generator=g) * 3
    k[-5:] *= 4
    v = torch.randn(T, H, 128, generator=g)
    q, k, v = (t.to(cuda).to(torch.bfloat16) for t in (q, k, v))
    out = ltxb.attention(q, k, v)
    torch.cuda.synchronize()
    assert ref.rel_rms(out.float().cpu(), _attn_ref(q, k, v)) < 1e-2


def test_attention_config1_sampled(cuda):
    """T = 28,160 (22x32x40), H = 32, q/k/v N(0,1) bf16 with
    the 3D RoPE pre-applied; 256 sampled query rows against dense f64."""
    import ltxb
    T, H = 28160, 32
    g = torch.Generator(device=cuda).manual_seed(1)
    q, k, v = (torch.randn(T, H, 128, generator=g, device=cuda) for _ in range(3))
    pos = oin.grid_positions(22, 32, 40)
    cos, sin = oin.rope_axes(pos, H)
    cos_t, sin_t = torch.from_numpy(cos).to(cuda), torch.from_numpy(sin).to(cuda)

    def rot(x):
        a, b = x[..., :64], x[..., 64:]
        return torch.cat([a * cos_t - b * sin_t, b * cos_t + a * sin_t], dim=-1)

    q, k = rot(q), rot(k)
    q, k, v = (t.to(torch.bfloat16).contiguous() for t in (q, k, v))
    out = ltxb.attention(q, k, v)
    torch.cuda.synchronize()
    rows = torch.from_numpy(np.random.default_rng(0).choice(T, 256, replace=False))
    want = _attn_ref(q[rows.to(cuda)], k, v)
    got = out[rows.to(cuda)].float().cpu()
    assert ref.rel_rms(got, want) < ATTN_TOL
    # cross-attention variant: K/V length 128
    out2 = ltxb.attention(q, k[:128].contiguous(), v[:128].contiguous())
    torch.cuda.synchronize()
    want2 = _attn_ref(q[rows.to(cuda)], k[:128], v[:128])
    assert ref.rel_rms(out2[rows.to(cuda)].float().cpu(), want2) < ATTN_TOL


@pytest.mark.parametrize("Tq,Tkv,H,splits", [(256, 1024, 2, 3), (300, 700, 3, 2), (130, 1000, 1, 8), (512, 2048, 4, 0),
                                             (3520, 28160, 2, 0)])
def test_attention_split(cuda, Tq, Tkv, H, splits):
    """Split-K/V attention (partial states merged by the combine kernel)
    against dense f64, and against the unsplit kernel."""
    import ltxb
    g = torch.Generator().manual_seed(Tq * 7 + Tkv)
    q = torch.randn(Tq, H, 128, generator=g).to(cuda).to(torch.bfloat16)
    k = torch.randn(Tkv, H, 128, generator=g).to(cuda).to(torch.bfloat16)
    v = torch.randn(Tkv, H, 128, generator=g).to(cuda).to(torch.bfloat16)
    gate = (2 * torch.sigmoid(torch.randn(Tq, H, generator=g))).to(cuda)
    got = ltxb.attention_split(q, k, v, gate, splits=splits)
    whole = ltxb.attention(q, k, v, gate)
    torch.cuda.synchronize()
    rows = torch.arange(0, Tq, max(1, Tq // 256))
    want = _attn_ref(q[rows.to(cuda)], k, v, gate[rows.to(cuda)])
    assert ref.rel_rms(got[rows.to(cuda)].float().cpu(), want) < ATTN_TOL
    assert ref.rel_rms(got.float().cpu(), whole.float().cpu()) < 2 * ATTN_TOL  # two independent bf16-P roundings
    assert ltxb.device_status() == ltxb.OK


def test_attention_split_errors(cuda):
    import ltxb
    q = torch.zeros(64, 1, 128, device=cuda, dtype=torch.bfloat16)
    small = torch.empty(16, dtype=torch.uint8, device=cuda)
    with pytest.raises(ltxb.LtxbError):
        ltxb.attention_split(q, q, q, splits=2, workspace=small)


def test_attention_deterministic(cuda):
    import ltxb
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(640, 4, 128, generator=g).to(cuda).to(torch.bfloat16) for _ in range(3))
    a = ltxb.attention(q, k, v)
    b = ltxb.attention(q, k, v)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_bounded_wait_expires_and_context_survives(cuda):
    """Failure detection without a fault: a kernel waits on an mbarrier that
    nothing arrives on; the bounded wait expires, the status word reports
    LTXB_ETIMEOUT with the self-test site, and after clearing it the same
    context runs kernels normally."""
    import time
    import ltxb
    assert ltxb.device_status() == ltxb.OK
    t0 = time.perf_counter()
    ltxb.selftest_wait(50_000)  # 50 ms
    rc, site = ltxb.device_status_site(clear=True)
    assert rc == ltxb.ETIMEOUT and site == ltxb.SELFTEST_SITE
    assert time.perf_counter() - t0 < 5.0
    assert ltxb.device_status() == ltxb.OK
    q = torch.randn(256, 2, 128, device=cuda).to(torch.bfloat16)
    out = ltxb.attention(q, q, q)
    torch.cuda.synchronize()
    assert ltxb.device_status() == ltxb.OK
    assert ref.rel_rms(out.float().cpu(), _attn_ref(q, q, q)) < ATTN_TOL
    with pytest.raises(ltxb.LtxbError):
        ltxb.selftest_wait(0)


@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 12288), (4096, 16384), (16384, 4096)])
def test_dq_gemm_config2_full_m_sampled_rows(cuda, K, N):
    """BASELINE config 2 at its full size: M = 28,160 bf16 N(0, 1) rows, W
    N(0, 0.02) with 0.5% of input channels x20, int8 g128 with bf16 scales,
    bf16 output -- through the expand-then-GEMM path the block uses. 256
    sampled rows (both edge tiles included) against f64 on the exactly
    dequantised weights; every row finite."""
    import ltxb
    M = 28160
    seed = 2000 + K + N
    w = oin.apply_outliers(oin.normal_f32(seed, "c2w", (N, K), 0.02), seed, "c2w")
    q, sc = ref.quantize_g128(w, scale_dtype="bf16")
    g = torch.Generator(device=cuda).manual_seed(seed)
    a = torch.randn(M, K, generator=g, device=cuda).to(torch.bfloat16)
    wq = torch.from_numpy(q).to(cuda)
    s = torch.from_numpy(sc.view(np.int16)).to(cuda).view(torch.bfloat16)
    out = ltxb.dq_gemm(a, wq, s, None, fused=False)
    torch.cuda.synchronize()
    assert ltxb.device_status() == ltxb.OK
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, 127, 128, M - 129, M - 128, M - 1], rng.choice(M, 250, replace=False)]))
    idx = torch.from_numpy(rows).to(cuda)
    got = out.index_select(0, idx).double().cpu()
    want = a.index_select(0, idx).double().cpu() @ torch.from_numpy(ref.dequant(q, sc)).T
    err = ref.rel_rms(got, want)
    print(f"\nconfig 2 K={K} N={N} M={M}: rel-RMS {err:.2e} on {len(rows)} rows")
    assert err < GEMM_TOL
    assert bool(torch.isfinite(out).all())
