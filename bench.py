#!/usr/bin/env python3
"""Benchmark: one int8-weight LTX-2.5 DiT block at T = 28,160 video tokens
(22x32x40 latent grid, D 4096, 32x128 heads, FFN 16384,
128 text tokens, int8 grouped-128 weights with bf16 scales for the q/k/v,
output and FFN projections), on 1..N B200s of one node with the tokens
sharded across ranks (sequence-parallel self-attention: head-parallel, each
rank attending its H/N heads over all tokens, with q/k/v and the attention
rows stored over NVLink straight into the other GPUs' memory).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torchrun (one rank per GPU). Rank 0 prints one JSON
line. A step is one block forward over all 28,160 tokens; `value` is the
whole-job throughput in TFLOP/s of algorithmic work (26.30 TFLOP per block).

`--impl reference` times the CPU restatement of the reference block
(oracle/, torch f32 on all host cores) on a bounded sample of the workload:
the reference itself is Zig on ZML/XLA and cannot be built on this machine.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "ltx-zml_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402

T_TOTAL, GRID, S, D, FF, H = 28160, (22, 32, 40), 128, 4096, 16384, 32
METRIC = "dit_block_tflops_28k_int8w"
# the library's default sequence-parallel exchange (LTXB_SP unset)
SP_DEFAULT = "peer"
# token counts of the CPU samples (latent grids with T % 1024 == 0, so the
# restated whileSdpa runs its production chunk of 1024 on every sample)
CPU_SAMPLE_GRIDS = ((8, 8, 16), (16, 8, 16), (12, 16, 16), (16, 16, 16))
SP_PARITY_TOL = 3e-3  # sequence-parallel output vs the 1-GPU output (rel-RMS)


def block_flops(T: int, s: int = S, d: int = D, ff: int = FF, h: int = H) -> float:
    """Algorithmic FLOPs of one block over T tokens (multiply-add = 2):
    self q/k/v/o 8TD^2, cross q/o 4TD^2, cross k/v 4SD^2, the two gate
    linears 4TDH, FFN 4TD.FF, self-attention 4T^2 D, cross-attention 4TSD."""
    return (8 * T * d * d + 4 * T * d * d + 4 * s * d * d + 4 * T * d * h + 4 * T * d * ff
            + 4 * T * T * d + 4 * T * s * d)


def phase_work(T_loc: int, T_all: int) -> dict:
    """(kind, amount per call) per library phase: FLOPs for tensor-core
    phases, bytes for the bandwidth-bound ones (minimum HBM traffic)."""
    return {
        "gemm_qkv1": ("tensor", 2 * T_loc * D * 3 * D),
        "gemm_gate1": ("tensor", 2 * T_loc * D * 32),
        "attn_self": ("tensor", 4 * T_loc * T_all * D),
        "gemm_o1": ("tensor", 2 * T_loc * D * D),
        "gemm_q2": ("tensor", 2 * T_loc * D * D),
        "gemm_gate2": ("tensor", 2 * T_loc * D * 32),
        "attn_cross": ("tensor", 4 * T_loc * S * D),
        "gemm_o2": ("tensor", 2 * T_loc * D * D),
        "gemm_ff1": ("tensor", 2 * T_loc * D * FF),
        "gemm_ff2": ("tensor", 2 * T_loc * FF * D),
        "prompt_kv": ("tensor", 2 * S * D * 2 * D),
        # x f32 read + n bf16 write
        "norm_msa": ("hbm", T_loc * D * (4 + 2)),
        "norm_ca": ("hbm", T_loc * D * (4 + 2)),
        "norm_mlp": ("hbm", T_loc * D * (4 + 2)),
        # q,k bf16 read + write, cos/sin f32 [T, H, 64] read
        "qk_norm_rope": ("hbm", T_loc * D * 2 * 4 + 2 * T_loc * H * 64 * 4),
        "qk_norm2": ("hbm", T_loc * D * 2 * 2),
    }


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return {"hbm": j["hbm_gbs"], "bf16": j["bf16_tflops"], "bf16_sustained": j["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        # the clock samples go to $LTXB_CLOCKS_DIR (e.g. a folder collected after
        # the run), else to the system temporary directory
        out_dir = os.environ.get("LTXB_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = pathlib.Path(out_dir) / f"clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in self.path.read_text().splitlines():
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                rows.append(dict(sm=float(p[1]), max=float(p[2]), power=float(p[3]), hw=p[5], hwt=p[6],
                                 swt=p[7], swp=p[8]))
            except ValueError:
                continue
        if not rows:
            return None
        load = [r for r in rows if r["power"] > 300] or rows
        reasons = set()
        for r in load:
            for k, nm in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                          ("swp", "sw_power_cap")):
                if r[k].lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["max"] for r in rows),
                "samples": len(load), "power_w_max": max(r["power"] for r in rows), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# synthetic config-3 block, generated on the GPU
# ---------------------------------------------------------------------------

def make_blob(device, seed: int = 0, block: int = 0):
    """Config-3 weights (ltxb.blobfmt.synthetic_block): N(0, 0.02) (norm
    weights 1 + N(0, 0.02), tables f32), int8 g128 for the extended set
    (q/k/v/o of both attentions and the FFN) after scaling 0.5% of input
    channels x20, symmetric absmax/127 scales rounded to bf16; packed in the
    reference blob format (name-sorted, 64-byte aligned)."""
    from ltxb import blobfmt
    return blobfmt.synthetic_block(device, D, FF, seed=seed, block=block)


def make_inputs(device, rank: int, world: int, seed: int = 0):
    """This rank's token slice of x [T, D], the 44/42/42 RoPE tables on the
    22x32x40 grid, tstab [1, 9, D] / tidx, ctx [128, D], pts2 [2, D]."""
    T = T_TOTAL // world
    r0 = rank * T
    g = torch.Generator(device=device)
    g.manual_seed(seed + 17)
    x_all = torch.randn(T_TOTAL, D, generator=g, device=device)
    x = x_all[r0:r0 + T].contiguous()
    del x_all
    g.manual_seed(seed + 18)
    ctx = torch.randn(S, D, generator=g, device=device)
    tstab = torch.randn(1, 9, D, generator=g, device=device) * 0.1
    pts2 = torch.randn(2, D, generator=g, device=device) * 0.1
    tidx = torch.zeros(T, dtype=torch.int32, device=device)
    f, hh, ww = GRID
    t = torch.arange(r0, r0 + T, device=device)
    pos = torch.stack([t // (hh * ww), (t // ww) % hh, t % ww], dim=1).double()
    ang = []
    for axis, dims in enumerate((44, 42, 42)):
        inv = 10000.0 ** (-2.0 * torch.arange(dims // 2, device=device, dtype=torch.float64) / dims)
        ang.append(pos[:, axis:axis + 1] * inv[None])
    a = torch.cat(ang, dim=1)
    cos = torch.cos(a).float()[:, None, :].expand(T, H, 64).contiguous()
    sin = torch.sin(a).float()[:, None, :].expand(T, H, 64).contiguous()
    return x, tstab, tidx, ctx, pts2, cos, sin


# ---------------------------------------------------------------------------
# CPU baseline: the oracle's block in torch f32 on the host cores
# ---------------------------------------------------------------------------

def cpu_block_sample(steps: int, warmup: int, budget_s: float = 1e9):
    """Times the CPU restatement (oracle.ltx_block_ref.QBlock, torch f32, all
    host threads) on config-3 architecture and int8 EXT weights at the token
    counts of CPU_SAMPLE_GRIDS (1,024 .. 4,096). One pass runs one block at
    each count; `warmup` untimed passes, then up to `steps` timed passes,
    stopping once `budget_s` seconds have been timed. Per count the median
    time is kept, and a + b T + c T^2 (linears and norms linear in T,
    self-attention quadratic) is fitted by least squares and evaluated at
    T = 28,160. Returns a dict with the fit, its residual and the
    extrapolated time and TFLOP/s of one full-size block."""
    from oracle import inputs as oin
    from oracle import ltx_block_ref as ref
    torch.set_num_threads(os.cpu_count() or 1)
    geom = ref.Geometry(d=D, ff=FF)
    bw = oin.make_weights(geom, 0, quant="int8", scale_dtype="bf16", qset=ref.Q8_FIELDS_EXT)
    blk = ref.QBlock(bw, torch.float32, qset=ref.Q8_FIELDS_EXT)
    samples = []
    for grid in CPU_SAMPLE_GRIDS:
        inp = oin.make_inputs(geom, grid=grid, s=S, seed=0, adaln="random")
        samples.append((grid[0] * grid[1] * grid[2], inp.torch(torch.float32)))
    times = {t: [] for t, _ in samples}
    with torch.no_grad():
        for _ in range(warmup):
            for _t, a in samples:
                blk.w_block_out(*a)
        t_all = time.perf_counter()
        done = 0
        while done < max(1, steps):
            for t, a in samples:
                t0 = time.perf_counter()
                blk.w_block_out(*a)
                times[t].append(time.perf_counter() - t0)
            done += 1
            if time.perf_counter() - t_all > budget_s:
                break
    ts = np.array([t for t, _ in samples], dtype=np.float64)
    med = np.array([statistics.median(times[int(t)]) for t in ts])
    A = np.stack([np.ones_like(ts), ts, ts * ts], axis=1)
    coef, *_ = np.linalg.lstsq(A, med, rcond=None)
    fit = A @ coef
    resid = float(np.max(np.abs(fit - med) / med))
    full_s = float(coef[0] + coef[1] * T_TOTAL + coef[2] * T_TOTAL * T_TOTAL)
    return {"tflops": block_flops(T_TOTAL) / full_s / 1e12, "ms_full": full_s * 1e3, "cores": torch.get_num_threads(),
            "passes": done, "samples_ms": {int(t): round(m * 1e3, 1) for t, m in zip(ts, med)},
            "fit_s": [float(c) for c in coef], "fit_max_rel_residual": resid,
            "sample_flops_tflops": {int(t): round(block_flops(int(t)) / m / 1e12, 3) for t, m in zip(ts, med)}}


def _cpu_sample_text(r: dict) -> str:
    a, b, c = r["fit_s"]
    return (f"oracle QBlock (torch f32, {r['cores']} host threads, int8 EXT weights, config-3 architecture) timed at "
            f"T = {', '.join(str(t) for t in r['samples_ms'])} (median ms {list(r['samples_ms'].values())}, "
            f"{r['passes']} passes); t(T) = {a:.3e} + {b:.3e} T + {c:.3e} T^2 s fitted by least squares "
            f"(max residual {100 * r['fit_max_rel_residual']:.1f}%), evaluated at T = {T_TOTAL}: {r['ms_full']:.0f} ms. "
            f"The reference's own whileSdpa would run chunk 16 at T = {T_TOTAL} (ltx/block.zig:105-108), not the "
            f"chunk 1024 timed here")


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    steps, warm = max(1, args.steps), max(0, args.warmup)
    # one step = one pass over the four sample token counts (~3-5 s on the
    # host); the timed passes stop after 120 s so the run ends within minutes
    r = cpu_block_sample(steps, warm, budget_s=120.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["tflops"], 4), "unit": "TFLOP/s", "n_gpus": world,
        "steps": r["passes"], "steps_requested": steps, "warmup": warm,
        "ms_per_step": round(r["ms_full"], 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "int8 DiT block, T=28160 (22x32x40), D=4096, S=128, FF=16384",
                   "sample": _cpu_sample_text(r)},
        "cpu_baseline": {"value": round(r["tflops"], 4), "unit": "TFLOP/s", "cores": r["cores"], "kind": "port",
                         "sample": _cpu_sample_text(r)},
        "e2e": {"value": round(r["tflops"], 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "fit": {"seconds_a_b_c": r["fit_s"], "max_rel_residual": round(r["fit_max_rel_residual"], 4),
                "samples_ms": r["samples_ms"], "sample_tflops": r["sample_flops_tflops"]},
        "note": "the reference (Zig on ZML/XLA) cannot be built here; its CPU path is timed through the "
                "oracle restatement; ms_per_step is the fitted time of one T=28160 block",
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# host placement: each rank's pinned buffers on its GPU's NUMA node
# ---------------------------------------------------------------------------

def _parse_cpulist(text: str) -> set:
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_host_locality(local_rank: int) -> dict:
    """The GPU's PCI address, NUMA node and local CPUs as sysfs reports them."""
    info = {"pci": None, "numa_node": None, "local_cpus": None}
    try:
        pr = torch.cuda.get_device_properties(local_rank)
        pci = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        info["pci"] = pci
        d = pathlib.Path("/sys/bus/pci/devices") / pci
        if (d / "numa_node").exists():
            info["numa_node"] = int((d / "numa_node").read_text())
        if (d / "local_cpulist").exists():
            info["local_cpus"] = (d / "local_cpulist").read_text().strip()
    except Exception:
        pass
    return info


def bind_to_gpu_numa(local_rank: int) -> dict:
    """Restricts this process to the GPU's local CPUs (when sysfs names a
    proper subset), so pinned host buffers allocated afterwards land on the
    GPU's NUMA node (pages are placed where they are first touched)."""
    info = gpu_host_locality(local_rank)
    info["bound"] = False
    try:
        allowed = os.sched_getaffinity(0)
        if info["local_cpus"]:
            cpus = _parse_cpulist(info["local_cpus"]) & allowed
            if cpus and cpus != allowed:
                os.sched_setaffinity(0, cpus)
                info["bound"] = True
        info["cpus_allowed"] = len(os.sched_getaffinity(0))
    except Exception:
        pass
    return info


def run_copy(args, rank: int, world: int, local_rank: int):
    """Host copies alone: every step copies this rank's x slice (T/N x D f32)
    from pinned host memory to the GPU and a block-output-sized buffer back,
    on two streams at once (the host pipe's steady state), with no compute.
    Prints the aggregate bytes per second over all ranks (max-over-ranks
    time), the bound the end-to-end number cannot beat."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    loc = bind_to_gpu_numa(local_rank) if not args.no_numa_bind else gpu_host_locality(local_rank)
    T = T_TOTAL // world
    x_host = torch.randn(T, D).pin_memory()
    out_host = torch.empty(T, D).pin_memory()
    x_dev = torch.empty(T, D, device=dev)
    out_dev = torch.randn(T, D, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def step():
        with torch.cuda.stream(s_in):
            x_dev.copy_(x_host, non_blocking=True)
        with torch.cuda.stream(s_out):
            out_host.copy_(out_dev, non_blocking=True)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3 / args.steps
    locs = [loc]
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        locs = [None] * world
        dist.all_gather_object(locs, loc)
    if rank == 0:
        nbytes = 2 * T * D * 4 * world
        print(json.dumps({"metric": "host_copy_aggregate_gbs", "value": round(nbytes / (ms * 1e-3) / 1e9, 1),
                          "unit": "GB/s", "n_gpus": world, "steps": args.steps, "ms_per_step": round(ms, 3),
                          "bytes_per_step_all_ranks": nbytes, "per_rank": f"{T} x {D} f32 in and out",
                          "numa_bind": not args.no_numa_bind, "ranks": locs}), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def run_ours(args, rank: int, world: int, local_rank: int):
    import ltxb
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    comm = None
    if world > 1:
        uid = [ltxb.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ltxb.Comm(uid[0], rank, world, local_rank)
    # the host pipe's pinned buffers go on this GPU's NUMA node
    locality = bind_to_gpu_numa(local_rank) if not args.no_numa_bind else gpu_host_locality(local_rank)
    data, ent = make_blob(dev)
    w = ltxb.build_quant_bufs(ltxb.Blob.from_bytes(data, ent), 0, qset=ltxb.QSET_EXT, hidden=D, ff=FF,
                              device=local_rank)
    del data
    blk = ltxb.QBlock(w, comm)
    x, tstab, tidx, ctx, pts2, cos, sin = make_inputs(dev, rank, world)
    T = x.shape[0]
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(args.warmup):
        blk.forward(x, tstab, tidx, ctx, pts2, cos, sin, out=out)
    barrier()
    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    ltxb.profile_collect(reset=True)
    ltxb.profile_enable(True)
    l0 = ltxb.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        blk.forward(x, tstab, tidx, ctx, pts2, cos, sin, out=out)
    e1.record(stream)
    barrier()
    launches = ltxb.launch_count() - l0
    ltxb.profile_enable(False)
    phases = ltxb.profile_collect(reset=True)
    ms = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop() if sampler else None
    status = ltxb.device_status(clear=True)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # end to end through the public API with host buffers: every step copies
    # its x from pinned host memory and its output back to pinned host memory
    # (ltxb_block_forward_host); the pipe overlaps step k's copies with the
    # compute of its neighbours
    x_host = x.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    pipe = blk.host_pipe(tstab, tidx, ctx, pts2, cos, sin, T)
    e2e_steps = max(3, min(args.steps, 10))
    pipe.forward(x_host, out_host)  # warm the pipe's buffers
    pipe.join()
    barrier()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(e2e_steps):
        pipe.forward(x_host, out_host)
    pipe.join()
    e3.record(stream)
    barrier()
    e2e_ms = e2.elapsed_time(e3) / e2e_steps
    e2e_ok = bool(torch.equal(out_host, out.cpu()))
    pipe.free()
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # After the timed regions: the structural check of the reference's
    # production pass (ltx/e2e_prod.zig:149-164) on the whole block output,
    # from the device statistics (statsOf); with N > 1 the ranks' outputs are
    # gathered and rank 0 compares them with a 1-GPU forward of the same
    # inputs (the ring-vs-direct gate of ltx/ring_dryrun.zig:288-313).
    full = out
    if dist is not None:
        gl = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gl, out)
        if rank == 0:
            full = torch.cat(gl, dim=0)
        del gl
    structural = sp_err = None
    if rank == 0:
        n_nan, ss, maxa = ltxb.stats_of(full)
        structural = {"nan": int(n_nan), "rms": round((ss / full.numel()) ** 0.5, 5), "max_abs": round(maxa, 4),
                      "tokens": full.shape[0], "source": "ltxb_stats (statsOf) on the whole output"}
        if dist is not None:
            x1, tstab1, tidx1, ctx1, pts21, cos1, sin1 = make_inputs(dev, 0, 1)
            one = ltxb.QBlock(w).forward(x1, tstab1, tidx1, ctx1, pts21, cos1, sin1)
            torch.cuda.synchronize()
            sp_err = float(((full.double() - one.double()).pow(2).sum() / one.double().pow(2).sum()).sqrt())
            del one, x1
    if dist is not None:
        dist.barrier()

    if rank == 0:
        pk = peaks()
        flops = block_flops(T_TOTAL)
        value = flops / (ms * 1e-3) / 1e12
        work = phase_work(T, T_TOTAL)
        steps = args.steps
        table = {}
        for nm, (tot_ms, nl, calls) in phases.items():
            per = tot_ms / max(1, calls)
            kind, amount = work.get(nm, ("other", 0))
            row = {"ms": round(per, 4), "share": round(tot_ms / (ms * steps), 4), "launches_per_call": nl // max(1, calls)}
            if kind == "tensor" and amount:
                row["tflops"] = round(amount / (per * 1e-3) / 1e12, 1)
            elif kind == "hbm" and amount:
                row["gbs"] = round(amount / (per * 1e-3) / 1e9, 1)
            table[nm] = row
        top = max(table, key=lambda k: table[k]["ms"]) if table else None
        roofline = None
        if top:
            kind, amount = work.get(top, ("tensor", 0))
            per_s = table[top]["ms"] * 1e-3
            if kind == "hbm":
                ach = amount / per_s / 1e9
                roofline = {"kernel": top, "bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm"],
                            "unit": "GB/s", "frac": round(ach / pk["hbm"], 4)}
            else:
                ach = amount / per_s / 1e12
                roofline = {"kernel": top, "bound": "tensor", "achieved": round(ach, 1), "peak": pk["bf16_sustained"],
                            "unit": "TFLOP/s", "frac": round(ach / pk["bf16_sustained"], 4),
                            "frac_of_burst_peak": round(ach / pk["bf16"], 4),
                            "algorithmic_per_launch": amount}
            tr = ROOT / "profiles" / "ncu_traffic.json"
            roofline["traffic"] = None
            if tr.exists():
                tj = json.loads(tr.read_text())
                if top in tj:
                    roofline["traffic"] = tj[top]["bytes_per_launch"]
            roofline["peak_source"] = pk["source"] + " (MEASURED_PEAKS.json; sustained for a kernel inside a long step)"
        env_sp = "ring" if os.environ.get("LTXB_SP_RING") == "1" else os.environ.get("LTXB_SP", "")
        if env_sp not in ("ring", "allgather", "alltoall", "peer"):
            env_sp = SP_DEFAULT if (SP_DEFAULT != "peer" or (comm is not None and comm.peer_mapped())) else "alltoall"
        sp_algo = {"ring": "send/recv ring of K/V shards", "allgather": "head-group pipelined K/V all-gather",
                   "peer": "head-parallel, q/k/v and attention rows stored straight into the other GPUs' memory"}.get(
            env_sp, "head-parallel all-to-all over NCCL send/recv: q/k/v to the ranks owning their heads, outputs back")
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "int8 DiT block, T=28160 (22x32x40), D=4096, 32x128 heads, S=128, FF=16384",
                       "weights": "int8 g128 (bf16 scales) q/k/v/o x2 + FFN; bf16 gates/norms/biases",
                       "parallelism": (f"sp{world} ({sp_algo} over NVLink)" if world > 1 else "single GPU"),
                       "tokens_per_rank": T, "l2": "inputs larger than L2 (x 461 MB f32, weights 0.7 GB)"},
            "frac_of_peak": round(value / world / pk["bf16"], 4),
            "frac_of_sustained_peak": round(value / world / pk["bf16_sustained"], 4),
            "roofline": roofline,
            "phases": table,
            "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": T_TOTAL * D * 4,
                    "d2h_bytes_per_step": T_TOTAL * D * 4, "steps": e2e_steps,
                    "api": "ltxb_block_forward_host (pinned host x in, block output out, copies pipelined)",
                    "output_matches_device_run": e2e_ok,
                    "host_placement": {"numa_bind": not args.no_numa_bind, "rank0": locality}},
            "structural": structural,
            "gpu_launches": launches,
            "gpu_launches_per_step": launches // max(1, args.steps),
            "clocks": clocks,
            "device_status": status,
        }
        if world == 1 and not args.no_cpu:
            try:
                os.sched_setaffinity(0, range(os.cpu_count() or 1))  # the CPU baseline gets every core
                # ~10-20 s of timed CPU work: passes over the four sample token counts
                r = cpu_block_sample(100, 1, budget_s=12.0)
                line["cpu_baseline"] = {"value": round(r["tflops"], 4), "unit": "TFLOP/s", "cores": r["cores"],
                                        "kind": "port", "sample": _cpu_sample_text(r)}
            except Exception as exc:  # the baseline is reported, never required
                line["cpu_baseline"] = {"value": None, "error": repr(exc)[:200]}
        if sp_err is not None:
            line["sp_rel_rms_vs_1gpu"] = sp_err
            line["sp_parity"] = {"rel_rms": sp_err, "tol": SP_PARITY_TOL,
                                 "how": "all ranks' outputs gathered after the timed region, compared on rank 0 "
                                        "with a 1-GPU ltxb_block_forward of the same inputs"}
        print(json.dumps(line), flush=True)
    w.free()
    if comm is not None:
        comm.free()
    if dist is not None:
        dist.destroy_process_group()
    if rank == 0 and ((sp_err is not None and not sp_err <= SP_PARITY_TOL) or (structural and structural["nan"])):
        print(f"parity failure: sp_rel_rms_vs_1gpu={sp_err}, structural={structural}", file=sys.stderr)
        return 1
    return 0


# ---------------------------------------------------------------------------
# the denoising loop (an extra measurement, not the driver's metric)
# ---------------------------------------------------------------------------

def make_core_blob(device, seed: int = 0):
    """Core-part weights N(0, 0.02) (bf16; scale_shift_table f32) in the blob format."""
    from ltxb import blobfmt
    g = torch.Generator(device=device)
    tensors = []
    for i, (name, spec, dt) in enumerate(blobfmt.CORE_TENSORS):
        shape = blobfmt.shape_of(spec, D)
        g.manual_seed(seed * 1000 + 500 + i)
        w = torch.randn(*shape, generator=g, device=device) * 0.02
        raw = w.cpu().numpy() if dt == "F32" else w.to(torch.bfloat16).view(torch.int16).cpu().numpy()
        tensors.append((name, dt, shape, raw.tobytes()))
    return blobfmt.pack(tensors)


def run_denoise(args, rank: int, world: int, local_rank: int):
    """ltxb_denoise_run over `--denoise-steps` distilled steps and `--blocks`
    int8 blocks (cycling over `--distinct` uploaded weight sets) at
    T = 28,160 on the 22x32x40 grid; prints one JSON line with the time per
    denoising step (max over ranks)."""
    import ltxb
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    comm = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        uid = [ltxb.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = ltxb.Comm(uid[0], rank, world, local_rank)
    sets = []
    for i in range(args.distinct):
        data, ent = make_blob(dev, seed=i)
        sets.append(ltxb.build_quant_bufs(ltxb.Blob.from_bytes(data, ent), 0, qset=ltxb.QSET_EXT, hidden=D, ff=FF,
                                          device=local_rank))
        del data
    blocks = [sets[b % len(sets)] for b in range(args.blocks)]
    cdata, cent = make_core_blob(dev)
    core = ltxb.Core(ltxb.Blob.from_bytes(cdata, cent), hidden=D, device=local_rank)
    T = T_TOTAL // world
    r0 = rank * T
    g = torch.Generator(device=dev)
    g.manual_seed(31)
    clean = torch.randn(T_TOTAL, 128, generator=g, device=dev)[r0:r0 + T].contiguous()
    noise = torch.randn(T_TOTAL, 128, generator=g, device=dev)[r0:r0 + T].contiguous()
    ctx = torch.randn(S, D, generator=g, device=dev)
    mask = torch.ones(T, device=dev)
    mask_values = torch.ones(1, device=dev)
    tidx = torch.zeros(T, dtype=torch.int32, device=dev)
    f, hh, ww = GRID
    t = torch.arange(r0, r0 + T, device=dev)
    pos = torch.stack([t // (hh * ww), (t // ww) % hh, t % ww], dim=1).float()
    cos, sin = ltxb.rope_tables(ltxb.ROPE_AXES, pos, H)
    sig = ltxb.sched_sigmas(1)[: args.denoise_steps + 1]
    latent = ltxb.sched_noise_init(clean, noise, mask, 1.0)
    stream = torch.cuda.current_stream()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    ltxb.denoise(core, blocks, sig[:2], latent.clone(), clean, mask, mask_values, tidx, ctx, cos, sin, comm)  # warm-up
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    ltxb.denoise(core, blocks, sig, latent, clean, mask, mask_values, tidx, ctx, cos, sin, comm)
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    finite = bool(torch.isfinite(latent).all().item())
    n = len(sig) - 1
    if rank == 0:
        flops = n * (args.blocks * block_flops(T_TOTAL) + 2 * 2.0 * T_TOTAL * D * 128)
        print(json.dumps({"metric": "denoise_step_ms", "value": round(ms / n, 3), "unit": "ms",
                          "higher_is_better": False, "n_gpus": world, "denoise_steps": n, "blocks": args.blocks,
                          "distinct_weight_sets": args.distinct, "tokens": T_TOTAL,
                          "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "latent_finite": finite,
                          "api": "ltxb_denoise_run (core parts + blocks + scheduler on the device)"}))
    for s_ in sets:
        s_.free()
    core.free()
    if comm is not None:
        comm.free()
    if dist is not None:
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--denoise", action="store_true",
                    help="instead of the block metric, time the whole denoising loop (ltxb_denoise_run)")
    ap.add_argument("--blocks", type=int, default=48, help="--denoise: blocks per step")
    ap.add_argument("--denoise-steps", type=int, default=8, help="--denoise: distilled steps (<= 8)")
    ap.add_argument("--distinct", type=int, default=4, help="--denoise: distinct uploaded weight sets")
    ap.add_argument("--copy-only", action="store_true",
                    help="instead of the block metric, time the host copies of the end-to-end pipe alone")
    ap.add_argument("--no-numa-bind", action="store_true",
                    help="leave each rank's pinned host buffers wherever the OS places them")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}; using WORLD_SIZE", file=sys.stderr)
    if T_TOTAL % world or (T_TOTAL // world) % 64:
        raise SystemExit(f"T={T_TOTAL} does not shard over {world} ranks")
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.denoise:
        return run_denoise(args, rank, world, local_rank)
    if args.copy_only:
        return run_copy(args, rank, world, local_rank)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
