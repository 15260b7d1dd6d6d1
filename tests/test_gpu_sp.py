"""Multi-GPU test of the sequence-parallel block (K/V all-gather + split-K/V
attention by default, the send/recv ring with LTXB_SP_RING=1, over NCCL):
tokens split across ranks, each rank holding its slice of x / tidx / RoPE
tables; the gathered outputs must match the f64 oracle of the whole block and
the single-GPU run of the library. Needs >= 2 GPUs (skipped otherwise).
NCCL's NVLink multicast is switched off for this test, as the pool requires
for multi-rank GPU tests."""

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import helpers
from oracle import ltx_block_ref as ref

pytestmark = pytest.mark.gpu

D, FF, S = 256, 512, 16


def _worker(rank, world, uid, grid, seed, mode, algo, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["LTXB_SP_RING"] = "1" if algo == "ring" else "0"
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-zml_b200"), os.path.join(root, "tests")]
    import ltxb
    import helpers as h
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        quant = "int8" if mode == "int8" else None
        geom, bw, data, ent, _ = h.weights_case(D, FF, seed, quant)
        inp = h.inputs_case(D, grid, S, seed, "axes", 3, "random")
        w = h.upload(data, ent, geom, ltxb.MODE_INT8 if quant else ltxb.MODE_BF16, device=rank)
        full = h.to_cuda(inp, dev)
        T_all = full[0].shape[0]
        T = T_all // world
        sl = slice(rank * T, (rank + 1) * T)
        x, tstab, tidx, ctx, pts2, cos, sin = full
        part = (x[sl].contiguous(), tstab, tidx[sl].contiguous(), ctx, pts2, cos[sl].contiguous(),
                sin[sl].contiguous())
        comm = ltxb.Comm(uid, rank, world, rank) if world > 1 else None
        blk = ltxb.Block(w, comm)
        out = blk.forward(*part)
        out2 = blk.forward(*part)  # second call reuses the ring buffers
        torch.cuda.synchronize()
        st = ltxb.device_status()
        q.put((rank, out.cpu().numpy(), bool(torch.equal(out, out2)), st, None))
        if comm is not None:
            comm.free()
        w.free()
    except Exception as exc:  # report, never hang the parent
        q.put((rank, None, False, -99, repr(exc)))


def _run(world, grid, seed, mode, algo="allgather"):
    import ltxb
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    uid = ltxb.Comm.unique_id()
    procs = [ctx.Process(target=_worker, args=(r, world, uid, grid, seed, mode, algo, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, arr, det, st, err = q.get(timeout=300)
            assert err is None, f"rank {r}: {err}"
            res[r] = (arr, det, st)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    for r, (_, det, st) in res.items():
        assert st == 0, f"rank {r}: device status {st}"
        assert det, f"rank {r}: repeated call differs"
    return np.concatenate([res[r][0] for r in range(world)], axis=0)


@pytest.mark.parametrize("algo", ["allgather", "ring"])
@pytest.mark.parametrize("mode,grid", [("bf16", (2, 4, 32)), ("int8", (3, 4, 16))])
def test_sp_block_matches_single_gpu_and_oracle(mode, grid, algo):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    seed = 3
    quant = "int8" if mode == "int8" else None
    geom, bw, data, ent, qset = helpers.weights_case(D, FF, seed, quant)
    inp = helpers.inputs_case(D, grid, S, seed, "axes", 3, "random")
    want = helpers.oracle_stages(bw, inp, qset if quant else None)["block_out"]
    sp = _run(2, grid, seed, mode, algo)
    single = _run(1, grid, seed, mode)
    assert ref.rel_rms(sp, want) < 5e-3
    assert ref.rel_rms(single, want) < 5e-3
    assert ref.rel_rms(sp, single) < 3e-3
