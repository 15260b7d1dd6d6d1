"""GPU test of ltxb_dq_gemm_noalloc, the int8 linear for callers that cannot
allocate device memory (their allocator owns the GPU, or they must not
allocate while running): through the C ABI, its output must match the
allocating entry point ltxb_dq_gemm on the same inputs, on two calls in a row
(the second with different weights, so the shared built-in scratch must be
overwritten, not reused). Collected last on purpose."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import inputs as oin
from oracle import ltx_block_ref as ref

pytestmark = pytest.mark.gpu

TOL = 4e-3  # the GEMM tolerance used by the other GPU tests (bf16 output)


def _noalloc_fn():
    import ltxb
    fn = ltxb.lib.ltxb_dq_gemm_noalloc
    vp = ctypes.c_void_p
    fn.restype = ctypes.c_int
    fn.argtypes = [vp, vp, vp, ctypes.c_int, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp]
    return fn


def _case(M, N, K, seed, scale_dtype, dev):
    w = oin.apply_outliers(oin.normal_f32(seed, "na_w", (N, K), 0.02), seed, "na_w")
    q, sc = ref.quantize_g128(w, scale_dtype=scale_dtype)
    a = torch.from_numpy(oin.normal_f32(seed, "na_a", (M, K), 1.0)).to(dev).to(torch.bfloat16)
    b = torch.from_numpy(oin.normal_f32(seed, "na_b", (N,), 0.02)).to(dev).to(torch.bfloat16)
    wq = torch.from_numpy(q).to(dev)
    s = (torch.from_numpy(sc.view(np.int16)).to(dev).view(torch.bfloat16) if scale_dtype == "bf16"
         else torch.from_numpy(sc).to(dev))
    return a, wq, s, b


def _run_noalloc(fn, a, wq, s, b):
    import ltxb
    M, K = a.shape
    N = wq.shape[0]
    out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    sdt = ltxb.DT_BF16 if s.dtype == torch.bfloat16 else ltxb.DT_F32
    rc = fn(a.data_ptr(), wq.data_ptr(), s.data_ptr(), sdt, b.data_ptr(), out.data_ptr(), M, N, K,
            torch.cuda.current_stream().cuda_stream)
    assert rc == ltxb.OK, ltxb.last_error()
    return out


def test_noalloc_matches_allocating_entry_point(cuda):
    import ltxb
    fn = _noalloc_fn()
    cases = [(384, 1024, 2048, 11, "f32"), (300, 4096, 4096, 12, "bf16")]  # the second fills the scratch
    got, want = [], []
    for M, N, K, seed, sdt in cases:  # two calls in a row on the shared scratch
        a, wq, s, b = _case(M, N, K, seed, sdt, cuda)
        got.append(_run_noalloc(fn, a, wq, s, b))
        want.append(ltxb.dq_gemm(a, wq, s, b, fused=False))
    torch.cuda.synchronize()
    assert ltxb.device_status() == ltxb.OK
    for g, w in zip(got, want):
        assert ref.rel_rms(g.float().cpu(), w.float().cpu()) <= TOL


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    import ltxb
    fn = _noalloc_fn()
    M, N, K = 16, 4096, 4224  # N * K * 2 exceeds LTXB_NOALLOC_SCRATCH_BYTES
    a = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda)
    wq = torch.zeros(N, K, dtype=torch.int8, device=cuda)
    s = torch.ones(N, K // 128, dtype=torch.float32, device=cuda)
    out = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    rc = fn(a.data_ptr(), wq.data_ptr(), s.data_ptr(), ltxb.DT_F32, None, out.data_ptr(), M, N, K,
            torch.cuda.current_stream().cuda_stream)
    assert rc == ltxb.EINVAL
    assert "scratch" in ltxb.last_error()


def test_noalloc_calls_allocate_no_device_memory(cuda):
    """The property the entry point exists for: once its first call on the
    device has looked up the scratch address (and the driver has loaded the
    kernels), further calls leave the device's free memory unchanged."""
    fn = _noalloc_fn()
    a, wq, s, b = _case(256, 2048, 4096, 13, "bf16", cuda)
    out = torch.empty(256, 2048, dtype=torch.bfloat16, device=cuda)
    st = torch.cuda.current_stream().cuda_stream
    import ltxb

    def call():
        rc = fn(a.data_ptr(), wq.data_ptr(), s.data_ptr(), ltxb.DT_BF16, b.data_ptr(), out.data_ptr(), 256, 2048,
                4096, st)
        assert rc == ltxb.OK, ltxb.last_error()

    call()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda)
    reserved0 = torch.cuda.memory_reserved(cuda)
    for _ in range(5):
        call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda)
    assert free1 == free0
    assert torch.cuda.memory_reserved(cuda) == reserved0
    assert ltxb.device_status() == ltxb.OK


def test_noalloc_rejects_bad_arguments_before_launching(cuda):
    """A call that ends in EINVAL (here a misaligned output) launches nothing,
    so it cannot overwrite the shared scratch under another caller's call."""
    import ltxb
    fn = _noalloc_fn()
    a, wq, s, b = _case(128, 1024, 2048, 14, "f32", cuda)
    out = torch.empty(128 * 1024 + 8, dtype=torch.bfloat16, device=cuda)
    n0 = ltxb.launch_count()
    rc = fn(a.data_ptr(), wq.data_ptr(), s.data_ptr(), ltxb.DT_F32, b.data_ptr(), out.data_ptr() + 2, 128, 1024, 2048,
            torch.cuda.current_stream().cuda_stream)
    assert rc == ltxb.EINVAL
    assert "aligned" in ltxb.last_error()
    assert ltxb.launch_count() == n0
