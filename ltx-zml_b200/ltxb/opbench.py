"""Operator micro-benchmarks of libltxb.so (one kernel family per run), for
timing and for sizing profiler captures:

    PYTHONPATH=ltx-zml_b200 python -m ltxb.opbench attention --T 8192 --H 8 --reps 3
    PYTHONPATH=ltx-zml_b200 python -m ltxb.opbench dq_gemm --M 8192 --N 4096 --K 4096 [--unfused]
    PYTHONPATH=ltx-zml_b200 python -m ltxb.opbench gemm --M 8192 --N 4096 --K 4096
    PYTHONPATH=ltx-zml_b200 python -m ltxb.opbench block --T 8192 --reps 3 [--phases]

`block` runs whole int8 blocks (BASELINE config-3 architecture: D 4096,
32 x 128 heads, FFN 16384, S 128, int8 g128 EXT weights with bf16 scales)
at T tokens, so every kernel of the block can be captured at a size chosen
for the profiler (`ncu -k regex:<kernel> -s <skip> -c 1`).

Inputs are seeded N(0, 1) activations and N(0, 0.02) weights generated on the
device; each run prints one line with the CUDA-event time per launch and the
algorithmic throughput.
"""

from __future__ import annotations

import argparse

import torch

from . import attention, dq_gemm, gemm_bf16, device_status, profile_collect, profile_enable


def _time(fn, reps: int) -> float:
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=("attention", "dq_gemm", "gemm", "block"))
    ap.add_argument("--T", type=int, default=8192)
    ap.add_argument("--Tkv", type=int, default=0)
    ap.add_argument("--H", type=int, default=8)
    ap.add_argument("--M", type=int, default=8192)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--unfused", action="store_true")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--phases", action="store_true", help="block: also print the per-phase device times")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    if a.op == "block":
        from . import QBlock, QSET_EXT, Blob, build_quant_bufs, blobfmt
        data, ent = blobfmt.synthetic_block(dev, 4096, 16384)
        w = build_quant_bufs(Blob.from_bytes(data, ent), 0, qset=QSET_EXT, hidden=4096, ff=16384)
        del data
        x = torch.randn(a.T, 4096, generator=g, device=dev)
        tstab = torch.randn(1, 9, 4096, generator=g, device=dev) * 0.1
        tidx = torch.zeros(a.T, dtype=torch.int32, device=dev)
        ctx = torch.randn(128, 4096, generator=g, device=dev)
        pts2 = torch.randn(2, 4096, generator=g, device=dev) * 0.1
        ang = torch.rand(a.T, 32, 64, generator=g, device=dev) * 6.283185307179586
        cos, sin = torch.cos(ang), torch.sin(ang)
        out = torch.empty_like(x)
        blk = QBlock(w)
        ms = _time(lambda: blk.forward(x, tstab, tidx, ctx, pts2, cos, sin, out=out), a.reps)
        T, D, S, FF = a.T, 4096, 128, 16384
        flop = 12 * T * D * D + 4 * S * D * D + 4 * T * D * 32 + 4 * T * D * FF + 4 * T * T * D + 4 * T * S * D
        print(f"block T={a.T}: {ms:.4f} ms/block {flop / ms / 1e9:.1f} TFLOP/s status={device_status()}")
        if a.phases:  # the library's per-phase device times over the same calls
            profile_collect(reset=True)
            profile_enable(True)
            _time(lambda: blk.forward(x, tstab, tidx, ctx, pts2, cos, sin, out=out), a.reps)
            profile_enable(False)
            ph = profile_collect(reset=True)
            print("phases (ms per block): " + " ".join(f"{k}={v[0] / max(v[2], 1):.4f}" for k, v in ph.items()))
        w.free()
        return 0
    if a.op == "attention":
        tkv = a.Tkv or a.T
        q = torch.randn(a.T, a.H, 128, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(tkv, a.H, 128, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(tkv, a.H, 128, generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)
        ms = _time(lambda: attention(q, k, v, out=out), a.reps)
        flop = 4.0 * a.T * tkv * a.H * 128
        print(f"attention T={a.T} Tkv={tkv} H={a.H}: {ms:.4f} ms/launch {flop / ms / 1e9:.1f} TFLOP/s "
              f"status={device_status()}")
    else:
        x = torch.randn(a.M, a.K, generator=g, device=dev).to(torch.bfloat16)
        w = torch.randn(a.N, a.K, generator=g, device=dev) * 0.02
        out = torch.empty(a.M, a.N, dtype=torch.bfloat16, device=dev)
        if a.op == "gemm":
            wb = w.to(torch.bfloat16)
            ms = _time(lambda: gemm_bf16(x, wb, out=out), a.reps)
        else:
            wg = w.view(a.N, a.K // 128, 128)
            sc = (wg.abs().amax(-1, keepdim=True) / 127.0).clamp_min(1e-12).to(torch.bfloat16)
            wq = torch.clamp(torch.round(wg / sc.float()), -128, 127).to(torch.int8).view(a.N, a.K)
            sc = sc.view(a.N, a.K // 128).contiguous()
            ws = None if not a.unfused else torch.empty(a.N * a.K * 2, dtype=torch.uint8, device=dev)
            ms = _time(lambda: dq_gemm(x, wq, sc, fused=not a.unfused, out=out, workspace=ws), a.reps)
        flop = 2.0 * a.M * a.N * a.K
        print(f"{a.op}{' unfused' if a.unfused else ''} M={a.M} N={a.N} K={a.K}: {ms:.4f} ms/launch "
              f"{flop / ms / 1e9:.1f} TFLOP/s status={device_status()}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
