"""GPU test of the staging ring's device path (ltxb_stage_*: the B200 form of
the reference's 2-slot pinned Ring, ltx/loader.zig:176-321): 48 schedule
positions over 4 distinct int8 blocks at the config-3 shape (D 4096, FFN
16384, int8 EXT weights, bf16 scales), staged by the reader thread through
two pinned (cudaHostAlloc) slots with first-touch digest checks and uploaded
with ltxb_stage_upload -- the cold start of a 48-block stack. The gate is the
reference's ring-vs-direct one (ltx/ring_dryrun.zig:288-313): every block
uploaded from a slot computes bit-for-bit what the same blob uploaded
directly (ltxb_weights_upload from the mapped blob) computes."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu

D, FF, N_DISTINCT, N_POS = 4096, 16384, 4, 48


def test_stage_cold_start_48_blocks_bitwise_equal_to_direct(tmp_path, cuda):
    import ltxb
    from ltxb import blobfmt
    dirs = []
    for i in range(N_DISTINCT):
        data, ent = blobfmt.synthetic_block(cuda, D, FF, seed=i, block=i)
        blobfmt.write_packed(tmp_path / f"block{i}", data, ent, block=i)
        dirs.append(tmp_path / f"block{i}")
        del data
    blobs = [ltxb.Blob.open(d) for d in dirs]
    schedule = [p % N_DISTINCT for p in range(N_POS)]
    stage = ltxb.Stage(blobs, schedule, pinned=True, verify=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    staged = [stage.upload(p, mode=ltxb.MODE_INT8, qset=ltxb.QSET_EXT, hidden=D, ff=FF, device=0)
              for p in range(N_POS)]
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    stats = stage.stats()
    stage.free()
    total = sum(len(blobs[b].data) for b in schedule)
    print(f"\nstaging ring cold start: {N_POS} blocks, {total / 1e9:.2f} GB in {dt:.2f} s "
          f"({total / dt / 1e9:.1f} GB/s incl. first-touch SHA-256 of {N_DISTINCT} blobs); stats {stats}")
    assert stats["staged_bytes"] == total
    direct = [ltxb.build_quant_bufs(b, i, qset=ltxb.QSET_EXT, hidden=D, ff=FF) for i, b in enumerate(blobs)]
    g = torch.Generator(device=cuda).manual_seed(5)
    T = 256
    x = torch.randn(T, D, generator=g, device=cuda)
    tstab = torch.randn(1, 9, D, generator=g, device=cuda) * 0.1
    tidx = torch.zeros(T, dtype=torch.int32, device=cuda)
    ctx = torch.randn(128, D, generator=g, device=cuda)
    pts2 = torch.randn(2, D, generator=g, device=cuda) * 0.1
    ang = torch.rand(T, 32, 64, generator=g, device=cuda) * 6.283185307179586
    cos, sin = torch.cos(ang), torch.sin(ang)
    want = [ltxb.QBlock(w).forward(x, tstab, tidx, ctx, pts2, cos, sin) for w in direct]
    for p, w in enumerate(staged):
        got = ltxb.QBlock(w).forward(x, tstab, tidx, ctx, pts2, cos, sin)
        assert torch.equal(got, want[schedule[p]]), f"position {p}: staged upload differs from the direct one"
    torch.cuda.synchronize()
    assert ltxb.device_status() == ltxb.OK
    for w in staged + direct:
        w.free()
