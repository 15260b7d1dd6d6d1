"""CPU tests of the sequence-parallel host logic with real multi-process ranks
over gloo:

* the head-parallel exchange (the library's default, by stores into the
  other ranks' memory, or over NCCL with LTXB_SP=alltoall): q/k/v blocks to
  the ranks owning their heads, attention over all tokens of the owned
  heads, output rows back to the ranks holding their tokens;
* the all-gather alternative: each rank all-gathers the K/V shards, splits
  the gathered K/V range and merges the per-split (m, l, O) partials the way
  the combine kernel does; the result must equal dense attention;
* the ring alternative: the library's ring schedule (ltxb_ring_step, the
  function the block's NCCL ring follows) drives a K/V shard exchange and
  each rank merges per-shard partials;
* a rank that dies before the exchange: the survivor's collective ends with
  an error within the process group's timeout."""

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ltx_block_ref as ref


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _partial(q, k, v):
    """(m, l, o) of one shard in log2 units, as the kernel's merge keeps them."""
    c = (1.0 / math.sqrt(q.shape[-1])) * 1.4426950408889634
    s = torch.einsum("qhd,khd->hqk", q, k) * c
    m = s.amax(-1)
    p = torch.exp2(s - m[..., None])
    return m, p.sum(-1), torch.einsum("hqk,khd->hqd", p, v)


def _ring_worker(rank, world, port, T, H, seed, result_q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-zml_b200")]
    import ltxb
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(seed)
        q_all = torch.randn(world * T, H, 128, generator=g, dtype=torch.float64)
        k_all = torch.randn(world * T, H, 128, generator=g, dtype=torch.float64)
        v_all = torch.randn(world * T, H, 128, generator=g, dtype=torch.float64)
        sl = slice(rank * T, (rank + 1) * T)
        q = q_all[sl]
        shards_k = {rank: k_all[sl].clone()}
        shards_v = {rank: v_all[sl].clone()}
        m = l = o = None
        for s in range(world):
            st = ltxb.ring_step(rank, world, s)
            cur = st["compute"]
            reqs = []
            if st["recv"] >= 0:
                rk = torch.empty_like(shards_k[cur])
                rv = torch.empty_like(shards_v[cur])
                reqs = [dist.isend(shards_k[cur], st["next"]), dist.isend(shards_v[cur], st["next"]),
                        dist.irecv(rk, st["prev"]), dist.irecv(rv, st["prev"])]
            mi, li, oi = _partial(q, shards_k[cur], shards_v[cur])
            if m is None:
                m, l, o = mi, li, oi
            else:
                mn = torch.maximum(m, mi)
                a, b = torch.exp2(m - mn), torch.exp2(mi - mn)
                l = l * a + li * b
                o = o * a[..., None] + oi * b[..., None]
                m = mn
            for r_ in reqs:
                r_.wait()
            if st["recv"] >= 0:
                shards_k[st["recv"]], shards_v[st["recv"]] = rk, rv
        out = (o / l[..., None]).permute(1, 0, 2)
        want = ref.sdpa_dense(q, k_all, v_all)
        seen = sorted(shards_k)
        result_q.put((rank, ref.rel_rms(out, want), seen))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ring_attention_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, 48, 2, 7, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, seen in res:
        assert err < 1e-12, (rank, err)
        assert seen == list(range(world)), "every rank must receive every shard exactly once"


def test_ring_schedule_properties():
    """Every rank attends to every shard exactly once; the shard received at
    step s is the one computed at step s+1; sends form a ring."""
    import ltxb
    for n in (1, 2, 4, 8):
        for r in range(n):
            steps = [ltxb.ring_step(r, n, s) for s in range(n)]
            assert sorted(st["compute"] for st in steps) == list(range(n))
            assert steps[0]["compute"] == r
            for s in range(n - 1):
                assert steps[s]["recv"] == steps[s + 1]["compute"]
            assert steps[-1]["recv"] == -1
            assert steps[0]["next"] == (r + 1) % n and steps[0]["prev"] == (r - 1) % n
            # what r receives at step s is what prev computed (and sent) at step s
            for s in range(n - 1):
                assert steps[s]["recv"] == ltxb.ring_step(steps[0]["prev"], n, s)["compute"]
    with pytest.raises(ltxb.LtxbError):
        ltxb.ring_step(2, 2, 0)


# ---------------------------------------------------------------------------
# the default sequence-parallel path: K/V all-gather + split-K/V combine
# ---------------------------------------------------------------------------

def _combine(parts):
    """The merge of attn_combine_kernel: m = max m_z, weights 2^(m_z - m)."""
    m = torch.stack([p[0] for p in parts]).amax(0)
    w = [torch.exp2(p[0] - m) for p in parts]
    l = sum(wz * p[1] for wz, p in zip(w, parts))
    o = sum(wz[..., None] * p[2] for wz, p in zip(w, parts))
    return o / l[..., None]


def _allgather_worker(rank, world, port, T, H, splits, seed, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(seed)
        q_all = torch.randn(world * T, H, 128, generator=g, dtype=torch.float64)
        k_all = torch.randn(world * T, H, 128, generator=g, dtype=torch.float64)
        v_all = torch.randn(world * T, H, 128, generator=g, dtype=torch.float64)
        sl = slice(rank * T, (rank + 1) * T)
        ks = [torch.empty(T, H, 128, dtype=torch.float64) for _ in range(world)]
        vs = [torch.empty(T, H, 128, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(ks, k_all[sl].contiguous())
        dist.all_gather(vs, v_all[sl].contiguous())
        k, v = torch.cat(ks), torch.cat(vs)
        n = k.shape[0]
        bounds = [z * n // splits for z in range(splits + 1)]
        parts = [_partial(q_all[sl], k[bounds[z]:bounds[z + 1]], v[bounds[z]:bounds[z + 1]]) for z in range(splits)]
        got = _combine(parts).permute(1, 0, 2)
        want = ref.sdpa_dense(q_all[sl], k_all, v_all).reshape(T, H, 128)
        result_q.put((rank, ref.rel_rms(got.numpy(), want.numpy()), torch.equal(k, k_all)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,splits", [(2, 3), (3, 4)])
def test_allgather_split_attention_gloo(world, splits):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_allgather_worker, args=(r, world, port, 40, 2, splits, 11, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, gathered in res:
        assert gathered, f"rank {rank}: gathered K differs from the global K"
        assert err < 1e-12, (rank, err)


def _failing_worker(rank, world, port, result_q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        result_q.put((rank, "raised"))
        raise SystemExit(3)  # this rank fails before the exchange
    import time
    t0 = time.time()
    try:
        out = [torch.empty(4) for _ in range(world)]
        dist.all_gather(out, torch.ones(4))
        result_q.put((rank, "completed"))
    except Exception as e:  # the survivor learns of the failure from the collective
        result_q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def test_rank_failure_surfaces_as_an_error_gloo():
    """A rank that dies before the K/V exchange: the other rank's collective
    ends with an error within the process group's timeout instead of
    hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    assert res[1] == "raised"
    assert res[0].startswith("error after"), res[0]


# ---------------------------------------------------------------------------
# the head-parallel exchange: q/k/v to the ranks owning their heads
# ---------------------------------------------------------------------------

def _alltoall_worker(rank, world, port, T, H, seed, result_q):
    """The block's SP_ALLTOALL arithmetic with real ranks: q/k/v [T, H, 128]
    of this rank's tokens are regrouped into [N][T][H/N, 128] (block p holds
    rank p's heads), one round of point-to-point messages sends block p to
    rank p and receives rank p's tokens for this rank's heads, which stack
    into [N T][H/N, 128] in global token order; attention over all tokens for
    the owned heads; the output rows [p T, (p+1) T) go back to rank p, whose
    received blocks are placed at head group p of its [T, H, 128] output."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(seed)
        full = [torch.randn(world * T, H, 128, generator=g, dtype=torch.float64) for _ in range(3)]
        sl = slice(rank * T, (rank + 1) * T)
        hn = H // world

        def exchange(blocks):  # blocks[p] goes to rank p; returns what each rank p sent here
            out = [None] * world
            reqs = []
            for p in range(world):
                if p == rank:
                    out[p] = blocks[p].clone()
                    continue
                out[p] = torch.empty(blocks[p].shape, dtype=blocks[p].dtype)
                reqs += [dist.isend(blocks[p].contiguous(), p), dist.irecv(out[p], p)]
            for r_ in reqs:
                r_.wait()
            return out

        mine = [x[sl] for x in full]  # this rank's tokens, every head
        recv = [exchange([x[:, p * hn:(p + 1) * hn] for p in range(world)]) for x in mine]
        q, k, v = (torch.cat(blocks, dim=0) for blocks in recv)  # [N T, H/N, 128]
        o = ref.sdpa_dense(q, k, v)  # this rank's heads, all tokens
        back = exchange([o[p * T:(p + 1) * T] for p in range(world)])
        got = torch.cat(back, dim=1)  # [T, H, 128]: head group p from rank p
        want = ref.sdpa_dense(full[0][sl], full[1], full[2])
        result_q.put((rank, ref.rel_rms(got.numpy(), want.numpy())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,T,H", [(2, 40, 2), (3, 24, 6)])
def test_alltoall_head_parallel_attention_gloo(world, T, H):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_alltoall_worker, args=(r, world, port, T, H, 13, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in res:
        assert err < 1e-12, (rank, err)
