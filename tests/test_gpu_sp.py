"""Multi-GPU test of the sequence-parallel block, with each of the library's
exchanges (LTXB_SP): the head-parallel exchange by stores into the other
ranks' memory (the default), the same exchange over NCCL send/recv, the K/V all-gather
with split-K/V attention, and the send/recv ring:
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
    if algo != "default":
        os.environ["LTXB_SP"] = algo
    os.environ["LTXB_SP_RING"] = "0"
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
        if comm is not None and algo in ("peer", "default") and not comm.peer_mapped():
            raise RuntimeError("peer windows not mapped")
        blk = ltxb.Block(w, comm)
        out = blk.forward(*part)
        # later calls reuse the exchange buffers (the peer windows alternate
        # two buffers by call parity: calls 1, 2, 3 use both, then the first again)
        out2 = blk.forward(*part)
        out3 = blk.forward(*part)
        torch.cuda.synchronize()
        st = ltxb.device_status()
        if comm is not None:
            comm.check()  # no error recorded on the group
        same = bool(torch.equal(out, out2)) and bool(torch.equal(out, out3))
        q.put((rank, out.cpu().numpy(), same, st, None))
        if comm is not None:
            comm.free()
        w.free()
    except Exception as exc:  # report, never hang the parent
        q.put((rank, None, False, -99, repr(exc)))


def _run(world, grid, seed, mode, algo="default"):
    return _spawn(world, _worker, (grid, seed, mode, algo))


def _spawn(world, target, args):
    """Runs target(rank, world, uid, *args, q) on `world` spawned ranks and
    returns the ranks' outputs concatenated along tokens."""
    import ltxb
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    uid = ltxb.Comm.unique_id()
    procs = [ctx.Process(target=target, args=(r, world, uid, *args, q)) for r in range(world)]
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


@pytest.mark.parametrize("algo", ["default", "alltoall", "allgather", "ring"])
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
    if algo in ("default", "alltoall"):  # every head computed as on one GPU
        assert np.array_equal(sp, single)


def _denoise_case():
    """Two int8 blocks, the core parts and three distilled steps at D 256 on a
    2x4x16 grid (128 tokens), a few tokens at mask value 0.5."""
    from oracle import core_ref as cr
    import ltxb
    grid = (2, 4, 16)
    T = grid[0] * grid[1] * grid[2]
    inp = helpers.inputs_case(D, grid, S, 4, "axes", 1, "random")
    rng = np.random.default_rng(9)
    clean = rng.standard_normal((T, 128)).astype(np.float32)
    noise = rng.standard_normal((T, 128)).astype(np.float32)
    mask_values = np.array([1.0, 0.5], dtype=np.float32)
    tidx = (np.arange(T) % 7 == 0).astype(np.int32)
    mask = mask_values[tidx]
    return dict(inp=inp, clean=clean, mask=mask, mask_values=mask_values, tidx=tidx,
                lat0=cr.noise_init(clean, noise, mask, 1.0), sig=ltxb.sched_sigmas(1)[:4])


def _denoise_worker(rank, world, uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-zml_b200"), os.path.join(root, "tests")]
    import ltxb
    import helpers as h
    from oracle import blob as oblob
    from oracle import core_ref as cr
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        c = _denoise_case()
        blocks = []
        for i in range(2):
            geom, _, data, ent, _ = h.weights_case(D, FF, 20 + i, "int8")
            blocks.append(h.upload(data, ent, geom, ltxb.MODE_INT8, device=rank))
        cdata, centries = oblob.pack(cr.core_tensors(cr.make_core_weights(D, 5)))
        cent = [dict(name=e.name, dtype=e.dtype, shape=e.shape, offset=e.offset, nbytes=e.nbytes) for e in centries]
        core = ltxb.Core(ltxb.Blob.from_bytes(cdata, cent), hidden=D, device=rank)
        T = c["lat0"].shape[0] // world
        sl = slice(rank * T, (rank + 1) * T)
        g = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        inp = c["inp"]
        lat = g(c["lat0"][sl])
        comm = ltxb.Comm(uid, rank, world, rank) if world > 1 else None
        ltxb.denoise(core, blocks, c["sig"], lat, g(c["clean"][sl]), g(c["mask"][sl]), g(c["mask_values"]),
                     g(c["tidx"][sl]), g(inp.ctx), g(inp.cos[sl]), g(inp.sin[sl]), comm=comm)
        torch.cuda.synchronize()
        q.put((rank, lat.cpu().numpy(), True, ltxb.device_status(), None))
        if comm is not None:
            comm.free()
        core.free()
        for b in blocks:
            b.free()
    except Exception as exc:  # report, never hang the parent
        q.put((rank, None, False, -99, repr(exc)))


def test_sp_denoise_loop_matches_single_gpu_and_oracle():
    """The whole denoising loop (core parts, two int8 blocks, the scheduler)
    with tokens split over 2 GPUs: the gathered latent after three steps
    against the single-GPU loop and the f64 oracle's trajectory (the
    reference's per-step 2e-3 gate, or the torch-bf16 loop's floor)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oracle import core_ref as cr
    sp = _spawn(2, _denoise_worker, ())
    single = _spawn(1, _denoise_worker, ())
    c = _denoise_case()
    inp = c["inp"]
    bws = [helpers.weights_case(D, FF, 20 + i, "int8")[1::3] for i in range(2)]
    run = lambda dtype: cr.denoise_ref(cr.CoreParts(cr.make_core_weights(D, 5)),
                                       [ref.QBlock(bw, dtype, qset=qs) for bw, qs in bws], c["sig"], c["lat0"],
                                       c["clean"], c["mask"], c["mask_values"], c["tidx"], inp.ctx, inp.cos,
                                       inp.sin, dtype=dtype)[-1]
    want = run(torch.float64)
    tol = max(2e-3, ref.rel_rms(run(torch.bfloat16), want))
    assert ref.rel_rms(sp, want) <= tol
    assert ref.rel_rms(single, want) <= tol
    assert ref.rel_rms(sp, single) < 3e-3


def _depart_worker(rank, world, uid, gone, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import sys
    import time
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-zml_b200"), os.path.join(root, "tests")]
    import ltxb
    import helpers as h
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        geom, bw, data, ent, _ = h.weights_case(D, FF, 3, "int8")
        inp = h.inputs_case(D, (2, 4, 32), S, 3, "axes", 3, "random")
        w = h.upload(data, ent, geom, ltxb.MODE_INT8, device=rank)
        full = h.to_cuda(inp, dev)
        T = full[0].shape[0] // world
        sl = slice(rank * T, (rank + 1) * T)
        x, tstab, tidx, ctx, pts2, cos, sin = full
        part = (x[sl].contiguous(), tstab, tidx[sl].contiguous(), ctx, pts2, cos[sl].contiguous(),
                sin[sl].contiguous())
        comm = ltxb.Comm(uid, rank, world, rank)
        ltxb.Block(w, comm).forward(*part)
        torch.cuda.synchronize()  # nothing of this rank is in flight from here on
        if rank == 1:
            gone.set()  # tells the survivor on the host (synchronous, unlike a queue put)
            os._exit(0)  # leaves between block calls without freeing anything
        if not gone.wait(timeout=120):  # the survivor learns of it on the host
            q.put((rank, None, "no departure signal"))
            return
        check = "ok"
        try:
            comm.check()
        except ltxb.LtxbError as e:
            check = f"error {e.code}"
        t0 = time.time()
        comm.abort()  # frees the group without waiting for the peer
        dt = time.time() - t0
        # the context stays usable: the whole block on this GPU alone
        out = ltxb.Block(w).forward(*full)
        torch.cuda.synchronize()
        q.put((rank, dict(check=check, abort_s=dt, status=ltxb.device_status(),
                          finite=bool(torch.isfinite(out).all())), None))
        w.free()
    except Exception as exc:  # report, never hang the parent
        q.put((rank, None, repr(exc)))


def test_departing_rank_survivor_aborts_and_continues():
    """A rank leaves between block calls (none of its kernels or collectives
    in flight) and says so on the host; the other rank's communicator check
    returns, ltxb_comm_abort returns promptly, and the same context then runs
    a single-GPU block normally -- the reference's Ring.abort / reader_err
    propagation (ltx/loader.zig:199-202, :240-247, :308-313) across ranks."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import ltxb
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    gone = ctx.Event()
    uid = ltxb.Comm.unique_id()
    procs = [ctx.Process(target=_depart_worker, args=(r, 2, uid, gone, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        r, s, err = q.get(timeout=300)  # only the survivor reports
        assert err is None, f"rank {r}: {err}"
        assert r == 0
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    assert procs[1].exitcode == 0, "the departing rank exits cleanly between block calls"
    print(f"\nsurvivor: check {s['check']}, abort {s['abort_s']:.3f} s, status {s['status']}")
    assert s["abort_s"] < 30.0
    assert s["status"] == 0 and s["finite"]
