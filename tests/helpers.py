"""Shared case builders for the parity tests: seeded weights and inputs from
the oracle's generators, packed into the reference's blob format, uploaded
through the library's C ABI, and the oracle's f64 answers for the same bytes."""

from __future__ import annotations

import functools

import numpy as np
import torch

from oracle import blob as oblob
from oracle import inputs as oin
from oracle import ltx_block_ref as ref


@functools.lru_cache(maxsize=8)
def weights_case(d: int, ff: int, seed: int, quant: str | None, scale_dtype: str = "f32", qext: bool = False):
    geom = ref.Geometry(d=d, ff=ff)
    qset = ref.Q8_FIELDS_EXT if qext else ref.Q8_FIELDS
    bw = oin.make_weights(geom, seed, quant=quant, scale_dtype=scale_dtype, qset=qset)
    data, entries = oblob.pack(oblob.block_tensors(bw, 0))
    ent = [dict(name=e.name, dtype=e.dtype, shape=e.shape, offset=e.offset, nbytes=e.nbytes) for e in entries]
    return geom, bw, data, ent, qset


@functools.lru_cache(maxsize=8)
def inputs_case(d: int, grid: tuple, s: int, seed: int, rope_layout: str = "axes", k_rows: int = 1,
                adaln: str = "mlp"):
    geom = ref.Geometry(d=d)
    return oin.make_inputs(geom, grid=grid, s=s, seed=seed, rope_layout=rope_layout, k_rows=k_rows, adaln=adaln)


def to_cuda(inp: oin.BlockInputs, device):
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
    return (f(inp.x), f(inp.tstab), f(inp.tidx), f(inp.ctx), f(inp.pts2), f(inp.cos), f(inp.sin))


def oracle_stages(bw, inp, quant_qset=None, dtype=torch.float64):
    blk = ref.QBlock(bw, dtype, qset=quant_qset) if quant_qset else ref.Block(bw, dtype)
    with torch.no_grad():
        return {k: v.to(torch.float64).numpy() for k, v in blk.staged(*inp.torch(dtype)).items()}


def upload(data, ent, geom, mode, qext=False, device=0):
    import ltxb
    b = ltxb.Blob.from_bytes(data, ent)
    if mode == ltxb.MODE_INT8:
        return ltxb.build_quant_bufs(b, 0, qset=ltxb.QSET_EXT if qext else ltxb.QSET_REF, hidden=geom.d,
                                     ff=geom.ff, device=device)
    return ltxb.build_block_bufs(b, 0, mode=mode, hidden=geom.d, ff=geom.ff, device=device)
