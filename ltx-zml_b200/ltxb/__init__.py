"""Python host mirror of the reference's block / loader interface over the
C ABI of libltxb.so (include/ltxb.h).

The reference drives its block through a compiled ZML executable
(ltx/e2e_prod.zig:297-395) and uploads weights with ltx/loader.zig. This
module gives the same operations, with the reference's names, on top of the
sm_100a library:

  Blob.open / check_layout / find_entry      ltx/loader.zig:45-129
  build_block_bufs / build_quant_bufs        ltx/loader.zig:133-172
  Block.s1NormMsa ... blockOut, wBlockOut     ltx/block.zig:248-353
  Block.wAttn1                               ltx/block.zig:274-276
  QBlock.qBlockOutAll / qBlockOut            ltx/block.zig:544-611
  Chain.chainB23 / chainB47 / wChainB47      ltx/block.zig:434-455
  attention (whileSdpa / sdpa)               ltx/block.zig:105-154, :234
  dq_gemm (linQ)                             ltx/block.zig:462-477

PyTorch provides device memory and streams only; every computation runs in
libltxb.so. If the library is missing this module raises at import -- there
is no fallback.
"""

from __future__ import annotations

import ctypes
import json
import pathlib

import numpy as np
import torch

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = _HERE / "libltxb.so"

OK = 0
EINVAL, ECUDA, ENOMEM, ELAYOUT, EMISSING, EDTYPE, ENCCL, ETIMEOUT, EUNSUPPORTED = range(-1, -10, -1)
DT_BF16, DT_F32, DT_I8 = 0, 1, 2
MODE_F32, MODE_BF16, MODE_INT8 = 0, 1, 2
QSET_REF, QSET_EXT, QSET_QKV = 0, 1, 2
VERIFY_BLOB, VERIFY_ENTRIES = 1, 2
STAGES = ["s1_norm_msa", "s1b_qnorm", "s2_attn1_nogate", "s3_attn1", "s4_after_sa", "s4_normed",
          "s5_ca_out", "s6_ff_in", "s7_ff_out", "block_out"]
_DT = {"BF16": DT_BF16, "F32": DT_F32, "I8": DT_I8}


class LtxbError(RuntimeError):
    """A failed library call: `.code` is the LTXB_E* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"ltxb error {code}: {msg}")
        self.code = code


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built (run `make -C ltx-zml_b200` or __graft_entry__.build())")
    lib = ctypes.CDLL(str(LIB_PATH))
    vp, i32, u64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_float
    sig = {
        "ltxb_init": (i32, [i32]),
        "ltxb_last_error": (ctypes.c_char_p, []),
        "ltxb_version": (ctypes.c_char_p, []),
        "ltxb_device_status": (i32, [i32, ctypes.POINTER(ctypes.c_uint32)]),
        "ltxb_selftest_wait": (i32, [ctypes.c_uint32, vp]),
        "ltxb_launch_count": (u64, []),
        "ltxb_profile_enable": (i32, [i32]),
        "ltxb_profile_collect": (i32, [i32, vp, i32, vp, vp, vp, i32]),
        "ltxb_blob_check_layout": (i32, [vp, i32, u64, ctypes.c_uint32]),
        "ltxb_blob_open": (i32, [ctypes.c_char_p, i32, ctypes.POINTER(vp)]),
        "ltxb_blob_close": (None, [vp]),
        "ltxb_blob_view": (i32, [vp, ctypes.POINTER(vp), ctypes.POINTER(u64), ctypes.POINTER(vp),
                                 ctypes.POINTER(i32), ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_int64)]),
        "ltxb_blob_find": (i32, [vp, ctypes.c_char_p, ctypes.POINTER(vp)]),
        "ltxb_blob_verify": (i32, [vp, i32]),
        "ltxb_sha256_hex": (None, [vp, u64, ctypes.c_char_p]),
        "ltxb_sha256_impl": (i32, [i32]),
        "ltxb_stage_create": (i32, [vp, i32, vp, i32, u64, i32, i32, ctypes.POINTER(vp)]),
        "ltxb_stage_acquire": (i32, [vp, i32, ctypes.POINTER(vp), ctypes.POINTER(u64), ctypes.c_uint32]),
        "ltxb_stage_release": (i32, [vp, i32]),
        "ltxb_stage_upload": (i32, [vp, i32, i32, i32, i32, i32, i32, i32, ctypes.c_uint32, ctypes.POINTER(vp)]),
        "ltxb_stage_get_stats": (i32, [vp, vp]),
        "ltxb_stage_abort": (None, [vp]),
        "ltxb_stage_free": (None, [vp]),
        "ltxb_weights_upload": (i32, [i32, vp, u64, vp, i32, i32, i32, i32, i32, i32, ctypes.POINTER(vp)]),
        "ltxb_weights_bytes": (u64, [vp]),
        "ltxb_weights_free": (None, [vp]),
        "ltxb_comm_id_bytes": (i32, []),
        "ltxb_comm_get_id": (i32, [vp]),
        "ltxb_comm_init": (i32, [vp, i32, i32, i32, ctypes.POINTER(vp)]),
        "ltxb_comm_free": (None, [vp]),
        "ltxb_comm_check": (i32, [vp]),
        "ltxb_comm_peer_mapped": (i32, [vp]),
        "ltxb_comm_abort": (None, [vp]),
        "ltxb_block_workspace_bytes": (u64, [vp, vp]),
        "ltxb_ring_step": (i32, [i32, i32, i32, vp, vp, vp, vp]),
        "ltxb_block_forward": (i32, [vp, vp, vp, vp]),
        "ltxb_block_stage": (i32, [vp, vp, vp, i32, vp, vp]),
        "ltxb_host_pipe_create": (i32, [vp, vp, vp, ctypes.POINTER(vp)]),
        "ltxb_block_forward_host": (i32, [vp, vp, vp, vp]),
        "ltxb_host_pipe_join": (i32, [vp, vp]),
        "ltxb_host_pipe_free": (None, [vp]),
        "ltxb_attention": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, f32, vp]),
        "ltxb_attention_split_workspace_bytes": (u64, [i32, i32, i32, i32]),
        "ltxb_rope_tables": (i32, [i32, vp, i32, i32, ctypes.c_double, vp, vp, vp]),
        "ltxb_core_upload": (i32, [i32, vp, u64, vp, i32, i32, ctypes.POINTER(vp)]),
        "ltxb_core_free": (None, [vp]),
        "ltxb_core_workspace_bytes": (u64, [vp, i32, i32]),
        "ltxb_core_sinusoid": (i32, [vp, i32, vp, vp]),
        "ltxb_core_adaln": (i32, [vp, vp, i32, vp, vp, vp, u64, vp]),
        "ltxb_core_pts2": (i32, [vp, vp, vp, vp, u64, vp]),
        "ltxb_core_patchify": (i32, [vp, vp, i32, vp, vp]),
        "ltxb_core_tail": (i32, [vp, vp, vp, i32, vp, i32, vp, vp, u64, vp]),
        "ltxb_sched_sigmas": (i32, [i32, vp, i32]),
        "ltxb_denoise_workspace_bytes": (u64, [vp, vp, vp]),
        "ltxb_denoise_run": (i32, [vp, vp, i32, vp, i32, vp, vp, vp]),
        "ltxb_sched_noise_init": (i32, [vp, vp, vp, i32, i32, f32, vp, vp]),
        "ltxb_sched_timesteps": (i32, [vp, i32, f32, vp, vp]),
        "ltxb_sched_step": (i32, [vp, vp, vp, vp, vp, i32, i32, f32, f32, vp, vp]),
        "ltxb_attention_split": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, f32, i32, vp, u64, vp]),
        "ltxb_dq_gemm": (i32, [vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, vp, u64, vp]),
        "ltxb_gemm_bf16": (i32, [vp, vp, vp, vp, i32, i32, i32, vp]),
        "ltxb_stats_workspace_bytes": (u64, []),
        "ltxb_stats": (i32, [vp, u64, vp, vp, u64, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _check(rc: int) -> None:
    if rc != OK:
        raise LtxbError(rc, lib.ltxb_last_error().decode(errors="replace"))


def last_error() -> str:
    return lib.ltxb_last_error().decode(errors="replace")


def version() -> str:
    return lib.ltxb_version().decode()


def device_status(clear: bool = True) -> int:
    """LTXB_OK or LTXB_ETIMEOUT (a bounded device wait expired). Syncs the device."""
    site = ctypes.c_uint32(0)
    return lib.ltxb_device_status(int(clear), ctypes.byref(site))


def device_status_site(clear: bool = True) -> tuple[int, int]:
    """(status, site code of the failing wait)."""
    site = ctypes.c_uint32(0)
    rc = lib.ltxb_device_status(int(clear), ctypes.byref(site))
    return rc, int(site.value)


SELFTEST_SITE = 0x7E0


def selftest_wait(limit_us: int, stream=None) -> None:
    """Run the bounded-wait self-test kernel (a wait that nothing satisfies)."""
    _check(lib.ltxb_selftest_wait(int(limit_us), _stream(stream)))


def launch_count() -> int:
    """Kernels libltxb.so has launched in this process."""
    return int(lib.ltxb_launch_count())


def profile_enable(on: bool = True) -> None:
    _check(lib.ltxb_profile_enable(int(on)))


def profile_collect(reset: bool = True) -> dict:
    """{phase: (total_ms, launches, calls)} accumulated since the last reset."""
    n = 64
    names = ctypes.create_string_buffer(n * 32)
    ms = (ctypes.c_double * n)()
    la = (ctypes.c_uint64 * n)()
    calls = (ctypes.c_int * n)()
    k = lib.ltxb_profile_collect(n, names, 32, ms, la, calls, int(reset))
    if k < 0:
        _check(k)
    out = {}
    for i in range(min(k, n)):
        nm = names.raw[i * 32:(i + 1) * 32].split(b"\0", 1)[0].decode()
        out[nm] = (ms[i], int(la[i]), calls[i])
    return out


def _ptr(t) -> int | None:
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous(), "tensors passed to libltxb must be contiguous CUDA tensors"
    return t.data_ptr()


def _stream(stream) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


# ---------------------------------------------------------------------------
# blob + loader (ltx/loader.zig)
# ---------------------------------------------------------------------------

class _Entry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 2), ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64)]


def _entry_array(entries):
    arr = (_Entry * len(entries))()
    keep = []
    for i, e in enumerate(entries):
        nm = e["name"].encode()
        keep.append(nm)
        arr[i].name = nm
        arr[i].dtype = _DT[e["dtype"]]
        arr[i].ndim = len(e["shape"])
        for j, d in enumerate(e["shape"][:2]):
            arr[i].shape[j] = d
        arr[i].offset = e["offset"]
        arr[i].nbytes = e["nbytes"]
    return arr, keep


def normalize_name(name: str) -> str:
    """ltx/loader.zig:102-119: '.' -> '_', '::' -> '_'."""
    return name.replace("::", "_").replace(".", "_")


class _BlobMapping:
    """Owns an ltxb_blob handle. The Blob and every view of its bytes hold a
    reference, so the mapping is released only when the last of them goes."""

    def __init__(self, handle):
        self.handle = handle

    def __del__(self):
        try:
            if self.handle:
                lib.ltxb_blob_close(self.handle)
                self.handle = None
        except Exception:
            pass


class Blob:
    """A packed block (blob.bin + blob_manifest.json, tools/pack_block.py).
    `Blob.open` goes through the library's native reader (ltxb_blob_open:
    manifest parse, size and layout checks, read-only mapping, SHA-256),
    like ltx/loader.zig:50-82; `data` is a uint8 view of the mapping."""

    def __init__(self, data, manifest: dict, mapping: _BlobMapping | None = None):
        self.data = data
        self.manifest = manifest
        self._map = mapping

    @classmethod
    def open(cls, directory, verify_digest: bool = False, verify_entries: bool = False) -> "Blob":
        """verify_digest: the whole blob against blob_sha256 (the loader's
        first-touch check, ltx/loader.zig:270-276); verify_entries: every
        entry against its own digest (parallel over host cores)."""
        h = ctypes.c_void_p()
        flags = (VERIFY_BLOB if verify_digest else 0) | (VERIFY_ENTRIES if verify_entries else 0)
        _check(lib.ltxb_blob_open(str(directory).encode(), flags, ctypes.byref(h)))
        mapping = _BlobMapping(h)
        p, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
        _check(lib.ltxb_blob_view(h, ctypes.byref(p), ctypes.byref(nbytes), None, None, None, None))
        n = int(nbytes.value)
        if n:
            buf = (ctypes.c_uint8 * n).from_address(p.value)
            buf._owner = mapping  # views of the bytes keep the mapping alive
            data = np.ctypeslib.as_array(buf)
        else:
            data = np.zeros(0, np.uint8)
        # the manifest's metadata (names, shapes, digests, provenance); the
        # native reader has checked the same file
        man = json.loads((pathlib.Path(directory) / "blob_manifest.json").read_text())
        return cls(data, man, mapping)

    def verify(self, entries: bool = False) -> None:
        """The digest checks of `open` on demand (ltxb_blob_verify)."""
        if self._map is None:
            raise LtxbError(EINVAL, "verify needs a blob from Blob.open")
        _check(lib.ltxb_blob_verify(self._map.handle, VERIFY_BLOB | (VERIFY_ENTRIES if entries else 0)))

    @classmethod
    def from_bytes(cls, data: bytes, entries: list[dict], align: int = 64, block: int = 0) -> "Blob":
        return cls(data, {"align": align, "block": block, "total_bytes": len(data), "entries": entries})

    def check_layout(self) -> None:
        """ltx/loader.zig:73-82 through the library's check."""
        arr, _keep = _entry_array(self.manifest["entries"])
        _check(lib.ltxb_blob_check_layout(ctypes.addressof(arr), len(arr), self.manifest["total_bytes"],
                                          self.manifest.get("align", 64)))

    def find_entry(self, want: str) -> dict:
        """ltx/loader.zig:122-129."""
        for e in self.manifest["entries"]:
            if normalize_name(e["name"]) == want:
                return e
        raise LtxbError(EMISSING, f"blob {self.manifest.get('block')}: no entry named {want}")


class _StageStats(ctypes.Structure):
    _fields_ = [("reader_parks", ctypes.c_uint64), ("consumer_parks", ctypes.c_uint64),
                ("copy_ns", ctypes.c_uint64), ("verify_ns", ctypes.c_uint64), ("staged_bytes", ctypes.c_uint64)]


class Stage:
    """ltxb_stage: a schedule of opened blobs streamed through two host slots
    by a reader thread (ltx/loader.zig:176-321's Ring). Take positions in
    order with `acquire` / `release`, or `upload` a block's weights."""

    def __init__(self, blobs: list, schedule: list, slot_bytes: int | None = None, pinned: bool = True,
                 verify: bool = True):
        if any(b._map is None for b in blobs):
            raise LtxbError(EINVAL, "Stage needs blobs from Blob.open")
        self._blobs = list(blobs)  # keeps the mappings alive
        handles = (ctypes.c_void_p * len(blobs))(*[b._map.handle.value for b in blobs])
        sched = (ctypes.c_int * len(schedule))(*schedule)
        if slot_bytes is None:
            slot_bytes = max([len(b.data) for b in blobs] + [1])
        h = ctypes.c_void_p()
        _check(lib.ltxb_stage_create(handles, len(blobs), sched, len(schedule), int(slot_bytes), int(pinned),
                                     int(verify), ctypes.byref(h)))
        self.handle = h
        self.schedule = list(schedule)

    def acquire(self, pos: int, timeout_ms: int = 60000) -> memoryview:
        """The staged bytes of schedule position `pos` (valid until release)."""
        p, n = ctypes.c_void_p(), ctypes.c_uint64()
        _check(lib.ltxb_stage_acquire(self.handle, pos, ctypes.byref(p), ctypes.byref(n), int(timeout_ms)))
        return memoryview((ctypes.c_uint8 * n.value).from_address(p.value)) if n.value else memoryview(b"")

    def release(self, pos: int) -> None:
        _check(lib.ltxb_stage_release(self.handle, pos))

    def upload(self, pos: int, mode: int = MODE_INT8, qset: int = QSET_REF, hidden: int = 4096, ff: int = 16384,
               device: int = 0, timeout_ms: int = 60000) -> "Weights":
        """buildQuantBufs / buildBlockBufs from the slot of position `pos`."""
        blk = self._blobs[self.schedule[pos]].manifest.get("block", 0)
        h = ctypes.c_void_p()
        _check(lib.ltxb_stage_upload(self.handle, pos, device, int(blk), mode, qset, hidden, ff, int(timeout_ms),
                                     ctypes.byref(h)))
        return Weights(h, mode, hidden, ff, device, qset)

    def stats(self) -> dict:
        s = _StageStats()
        _check(lib.ltxb_stage_get_stats(self.handle, ctypes.byref(s)))
        return {k: int(getattr(s, k)) for k, _ in _StageStats._fields_}

    def abort(self) -> None:
        lib.ltxb_stage_abort(self.handle)

    def free(self) -> None:
        if self.handle:
            lib.ltxb_stage_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Weights:
    """Device-resident weights of one block (an `ltxb_weights*`)."""

    def __init__(self, handle, mode, hidden, ff, device, qset=QSET_REF):
        self.handle = handle
        self.mode = mode
        self.qset = qset
        self.D = hidden
        self.FF = ff
        self.H = hidden // 128
        self.device = device

    @property
    def nbytes(self) -> int:
        return lib.ltxb_weights_bytes(self.handle)

    def free(self) -> None:
        if self.handle:
            lib.ltxb_weights_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _upload(blob: Blob, block_idx: int, mode: int, qset: int, hidden: int, ff: int, device: int) -> Weights:
    host = np.frombuffer(blob.data, dtype=np.uint8)
    arr, _keep = _entry_array(blob.manifest["entries"])
    h = ctypes.c_void_p()
    _check(lib.ltxb_weights_upload(device, host.ctypes.data, host.size, ctypes.addressof(arr), len(arr),
                                   block_idx, mode, qset, hidden, ff, ctypes.byref(h)))
    return Weights(h, mode, hidden, ff, device, qset)


def build_block_bufs(blob: Blob, block_idx: int, mode: int = MODE_BF16, hidden: int = 4096, ff: int = 16384,
                     device: int = 0) -> Weights:
    """ltx/loader.zig:133-144: the 28 base tensors of a block, device-resident."""
    return _upload(blob, block_idx, mode, QSET_REF, hidden, ff, device)


def build_quant_bufs(blob: Blob, block_idx: int, qset: int = QSET_REF, hidden: int = 4096, ff: int = 16384,
                     device: int = 0) -> Weights:
    """ltx/loader.zig:158-172: int8 g128 pairs for the quantised linears
    (QSET_REF: qBlockOutAll's set; QSET_EXT: + output projections; QSET_QKV:
    q/k/v only, qBlockOut's set)."""
    return _upload(blob, block_idx, MODE_INT8, qset, hidden, ff, device)


# ---------------------------------------------------------------------------
# core parts and scheduler (ltx/core_parts.zig, ltx/scheduler.zig)
# ---------------------------------------------------------------------------

class Core:
    """Device-resident core parts (`ltxb_core*`): CoreParts' methods on the GPU."""

    def __init__(self, blob: Blob, hidden: int = 4096, device: int = 0):
        host = np.frombuffer(blob.data, dtype=np.uint8)
        arr, _keep = _entry_array(blob.manifest["entries"])
        h = ctypes.c_void_p()
        _check(lib.ltxb_core_upload(device, host.ctypes.data, host.size, ctypes.addressof(arr), len(arr), hidden,
                                    ctypes.byref(h)))
        self.handle, self.D, self.device = h, hidden, device

    def free(self) -> None:
        if self.handle:
            lib.ltxb_core_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def _ws(self, T: int, K: int, dev):
        n = lib.ltxb_core_workspace_bytes(self.handle, T, K)
        return torch.empty(max(int(n), 1), dtype=torch.uint8, device=dev)

    @staticmethod
    def sinusoid(t, stream=None) -> torch.Tensor:
        t = t.contiguous().float()
        out = torch.empty(t.numel(), 256, dtype=torch.float32, device=t.device)
        _check(lib.ltxb_core_sinusoid(_ptr(t), t.numel(), _ptr(out), _stream(stream)))
        return out

    def adaln(self, t, stream=None):
        """t [K] -> (embedded_timestep [K, D], ts9 [K, 9, D])."""
        t = t.contiguous().float()
        K = t.numel()
        emb = torch.empty(K, self.D, dtype=torch.float32, device=t.device)
        ts9 = torch.empty(K, 9, self.D, dtype=torch.float32, device=t.device)
        ws = self._ws(0, K, t.device)
        _check(lib.ltxb_core_adaln(self.handle, _ptr(t), K, _ptr(emb), _ptr(ts9), _ptr(ws), ws.numel(),
                                   _stream(stream)))
        return emb, ts9

    def pts2(self, sigma, stream=None) -> torch.Tensor:
        """sigma (one-element device tensor) -> pts2 [2, D]."""
        sigma = sigma.contiguous().float()
        out = torch.empty(2, self.D, dtype=torch.float32, device=sigma.device)
        ws = self._ws(0, 1, sigma.device)
        _check(lib.ltxb_core_pts2(self.handle, _ptr(sigma), _ptr(out), _ptr(ws), ws.numel(), _stream(stream)))
        return out

    def patchify(self, latent, stream=None) -> torch.Tensor:
        latent = latent.contiguous().float()
        out = torch.empty(latent.shape[0], self.D, dtype=torch.float32, device=latent.device)
        _check(lib.ltxb_core_patchify(self.handle, _ptr(latent), latent.shape[0], _ptr(out), _stream(stream)))
        return out

    def tail(self, x, emb, tidx=None, stream=None) -> torch.Tensor:
        """tailFromEmb: x [T, D], emb [K, D] with tidx [T] (or emb [T, D]) -> velocity [T, 128].
        A tidx outside [0, K) reads row 0, as the block's table select does."""
        T = x.shape[0]
        out = torch.empty(T, 128, dtype=torch.float32, device=x.device)
        ws = self._ws(T, 1, x.device)
        _check(lib.ltxb_core_tail(self.handle, _ptr(x), _ptr(emb), emb.shape[0], _ptr(tidx), T, _ptr(out), _ptr(ws), ws.numel(),
                                  _stream(stream)))
        return out


def sched_sigmas(stage: int) -> np.ndarray:
    n = lib.ltxb_sched_sigmas(stage, None, 0)
    if n < 0:
        _check(n)
    out = np.zeros(n, dtype=np.float32)
    _check(min(0, lib.ltxb_sched_sigmas(stage, out.ctypes.data, n)))
    return out


def sched_noise_init(clean, noise, mask, noise_scale: float, out=None, stream=None) -> torch.Tensor:
    T, C = clean.shape
    out = torch.empty_like(clean) if out is None else out
    _check(lib.ltxb_sched_noise_init(_ptr(clean), _ptr(noise), _ptr(mask), T, C, float(noise_scale), _ptr(out),
                                     _stream(stream)))
    return out


def sched_timesteps(mask, sigma: float, out=None, stream=None) -> torch.Tensor:
    out = torch.empty_like(mask) if out is None else out
    _check(lib.ltxb_sched_timesteps(_ptr(mask), mask.numel(), float(sigma), _ptr(out), _stream(stream)))
    return out


def sched_step(x, velocity, ts, clean, mask, sigma: float, sigma_next: float, out=None, stream=None) -> torch.Tensor:
    T, C = x.shape
    out = torch.empty_like(x) if out is None else out
    _check(lib.ltxb_sched_step(_ptr(x), _ptr(velocity), _ptr(ts), _ptr(clean), _ptr(mask), T, C, float(sigma),
                               float(sigma_next), _ptr(out), _stream(stream)))
    return out


# ---------------------------------------------------------------------------
# communicator (sequence parallelism)
# ---------------------------------------------------------------------------

def ring_step(rank: int, nranks: int, step: int) -> dict:
    """The library's ring schedule (ltxb_ring_step): which K/V shard this rank
    attends to at `step`, which shard it receives meanwhile (-1 on the last
    step), and its ring neighbours."""
    out = [ctypes.c_int() for _ in range(4)]
    _check(lib.ltxb_ring_step(rank, nranks, step, *[ctypes.byref(o) for o in out]))
    return dict(compute=out[0].value, recv=out[1].value, next=out[2].value, prev=out[3].value)


class Comm:
    """Sequence-parallel group (one rank per GPU): an NCCL communicator plus,
    with 2..8 ranks in separate processes, every rank's peer-memory window
    mapped in every other rank (the default head-parallel exchange)."""

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(lib.ltxb_comm_id_bytes())
        _check(lib.ltxb_comm_get_id(buf))
        return buf.raw

    def __init__(self, uid: bytes, rank: int, nranks: int, device: int):
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(uid, len(uid))
        _check(lib.ltxb_comm_init(buf, rank, nranks, device, ctypes.byref(h)))
        self.handle, self.rank, self.nranks = h, rank, nranks

    def peer_mapped(self) -> bool:
        """True when every rank mapped every other rank's memory window, so
        the head-parallel exchange can run as stores into peer memory."""
        return bool(lib.ltxb_comm_peer_mapped(self.handle))

    def free(self):
        if self.handle:
            lib.ltxb_comm_free(self.handle)
            self.handle = None

    def check(self) -> None:
        """Raises LtxbError(ENCCL) if NCCL has recorded an error on the group."""
        _check(lib.ltxb_comm_check(self.handle))

    def abort(self):
        """Frees the group without waiting for its transfers (a peer is gone)."""
        if self.handle:
            lib.ltxb_comm_abort(self.handle)
            self.handle = None


# ---------------------------------------------------------------------------
# the block
# ---------------------------------------------------------------------------

class _Config(ctypes.Structure):
    _fields_ = [("T", ctypes.c_int32), ("S", ctypes.c_int32), ("K", ctypes.c_int32), ("mode", ctypes.c_int32),
                ("sp_rank", ctypes.c_int32), ("sp_size", ctypes.c_int32), ("comm", ctypes.c_void_p)]


class _IO(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("out", ctypes.c_void_p), ("tstab", ctypes.c_void_p),
                ("tidx", ctypes.c_void_p), ("ctx", ctypes.c_void_p), ("pts2", ctypes.c_void_p),
                ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_uint64)]


class _DenoiseIO(ctypes.Structure):
    _fields_ = [("latent", ctypes.c_void_p), ("clean", ctypes.c_void_p), ("mask", ctypes.c_void_p),
                ("mask_values", ctypes.c_void_p), ("tidx", ctypes.c_void_p), ("ctx", ctypes.c_void_p),
                ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_uint64)]


def denoise(core: "Core", blocks: list, sigmas, latent, clean, mask, mask_values, tidx, ctx, cos, sin,
            comm: "Comm | None" = None, stream=None):
    """The denoising loop of ltx/e2e_denoise.zig:218-336 on the device
    (ltxb_denoise_run): len(sigmas) - 1 steps over all `blocks`; `latent`
    [T, 128] f32 is updated in place and returned."""
    sig = np.ascontiguousarray(np.asarray(sigmas, dtype=np.float32))
    T = latent.shape[0]
    w0 = blocks[0]
    cfg = _Config(T, ctx.shape[0], mask_values.numel(), w0.mode, comm.rank if comm else 0,
                  comm.nranks if comm else 1, comm.handle if comm else None)
    need = lib.ltxb_denoise_workspace_bytes(core.handle, w0.handle, ctypes.byref(cfg))
    ws = torch.empty(int(need), dtype=torch.uint8, device=latent.device)
    io = _DenoiseIO(_ptr(latent), _ptr(clean), _ptr(mask), _ptr(mask_values), _ptr(tidx), _ptr(ctx), _ptr(cos),
                    _ptr(sin), _ptr(ws), ws.numel())
    handles = (ctypes.c_void_p * len(blocks))(*[b.handle for b in blocks])
    _check(lib.ltxb_denoise_run(core.handle, handles, len(blocks), sig.ctypes.data, len(sig) - 1, ctypes.byref(io),
                                ctypes.byref(cfg), _stream(stream)))
    return latent


class Block:
    """A block bound to device weights: the reference's traced methods
    (ltx/block.zig:248-353). Inputs are CUDA tensors:
    x [T, D] f32, tstab [K, 9, D] f32, tidx [T] int32, ctx [S, D] f32,
    pts2 [2, D] f32, cos/sin [T, H, 64] f32."""

    def __init__(self, weights: Weights, comm: Comm | None = None):
        self.w = weights
        self.comm = comm
        self._ws = None

    def _cfg(self, T, S, K):
        c = _Config(T, S, K, self.w.mode, self.comm.rank if self.comm else 0,
                    self.comm.nranks if self.comm else 1, self.comm.handle if self.comm else None)
        return c

    def workspace_bytes(self, T: int, S: int, K: int = 1) -> int:
        c = self._cfg(T, S, K)
        return lib.ltxb_block_workspace_bytes(self.w.handle, ctypes.byref(c))

    def _workspace(self, nbytes: int, device) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < nbytes or self._ws.device != device:
            self._ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
        return self._ws

    def _io(self, x, tstab, tidx, ctx, pts2, cos, sin, out):
        T, S, K = x.shape[0], ctx.shape[0], tstab.shape[0]
        c = self._cfg(T, S, K)
        nbytes = lib.ltxb_block_workspace_bytes(self.w.handle, ctypes.byref(c))
        ws = self._workspace(nbytes, x.device)
        base = ws.data_ptr()
        aligned = (base + 255) & ~255
        io = _IO(_ptr(x), _ptr(out), _ptr(tstab), _ptr(tidx), _ptr(ctx), _ptr(pts2), _ptr(cos), _ptr(sin),
                 aligned, ws.numel() - (aligned - base))
        return c, io

    def forward(self, x, tstab, tidx, ctx, pts2, cos, sin, out=None, stream=None) -> torch.Tensor:
        """ltxb_block_forward: the whole block with blockwise attention."""
        out = torch.empty_like(x) if out is None else out
        c, io = self._io(x, tstab, tidx, ctx, pts2, cos, sin, out)
        _check(lib.ltxb_block_forward(self.w.handle, ctypes.byref(io), ctypes.byref(c), _stream(stream)))
        return out

    def stage(self, stage: int | str, x, tstab, tidx, ctx, pts2, cos, sin, stream=None) -> torch.Tensor:
        si = STAGES.index(stage) if isinstance(stage, str) else stage
        out = torch.empty_like(x)
        scratch = torch.empty_like(x)
        c, io = self._io(x, tstab, tidx, ctx, pts2, cos, sin, scratch)
        _check(lib.ltxb_block_stage(self.w.handle, ctypes.byref(io), ctypes.byref(c), si, _ptr(out),
                                    _stream(stream)))
        return out

    def host_pipe(self, tstab, tidx, ctx, pts2, cos, sin, T: int) -> "HostPipe":
        """A pipelined host-buffer runner bound to these device tables."""
        return HostPipe(self, tstab, tidx, ctx, pts2, cos, sin, T)

    # the reference's method names (ltx/block.zig:248-353)
    def blockOut(self, x, tstab, tidx, ctx, pts2, cos, sin):
        return self.forward(x, tstab, tidx, ctx, pts2, cos, sin)

    def wBlockOut(self, x, tstab, tidx, ctx, pts2, cos, sin):
        """Same function as blockOut: attention here is always the blockwise
        online softmax, which the reference gates against dense at 1e-5."""
        return self.forward(x, tstab, tidx, ctx, pts2, cos, sin)

    def wAttn1(self, x, tstab, tidx, cos, sin, ctx=None, pts2=None):
        """ltx/block.zig:274-276: s3Attn1 with the blockwise softmax -- the
        same call as s3Attn1 here. The stage reads neither ctx nor pts2; rows
        of x stand in for them unless given."""
        return self.s3Attn1(x, tstab, tidx, x[:1] if ctx is None else ctx, x[:2] if pts2 is None else pts2, cos, sin)

    def s1NormMsa(self, *a):
        return self.stage("s1_norm_msa", *a)

    def s1bQnorm(self, *a):
        return self.stage("s1b_qnorm", *a)

    def s2Attn1NoGate(self, *a):
        return self.stage("s2_attn1_nogate", *a)

    def s3Attn1(self, *a):
        return self.stage("s3_attn1", *a)

    def s4AfterSa(self, *a):
        return self.stage("s4_after_sa", *a)

    def s4Normed(self, *a):
        return self.stage("s4_normed", *a)

    def s5CaOut(self, *a):
        return self.stage("s5_ca_out", *a)

    def s6FfIn(self, *a):
        return self.stage("s6_ff_in", *a)

    def s7FfOut(self, *a):
        return self.stage("s7_ff_out", *a)


class HostPipe:
    """ltxb_host_pipe: x from pinned host memory in, block output to pinned
    host memory out, with the copies of neighbouring calls overlapping the
    compute (see include/ltxb.h)."""

    def __init__(self, blk: Block, tstab, tidx, ctx, pts2, cos, sin, T: int):
        self.blk = blk
        self._keep = (tstab, tidx, ctx, pts2, cos, sin)
        S, K = ctx.shape[0], tstab.shape[0]
        c = blk._cfg(T, S, K)
        nbytes = lib.ltxb_block_workspace_bytes(blk.w.handle, ctypes.byref(c))
        self._ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=ctx.device)
        base = self._ws.data_ptr()
        aligned = (base + 255) & ~255
        io = _IO(None, None, _ptr(tstab), _ptr(tidx), _ptr(ctx), _ptr(pts2), _ptr(cos), _ptr(sin), aligned,
                 self._ws.numel() - (aligned - base))
        h = ctypes.c_void_p()
        _check(lib.ltxb_host_pipe_create(blk.w.handle, ctypes.byref(c), ctypes.byref(io), ctypes.byref(h)))
        self.handle = h

    def forward(self, x_host: torch.Tensor, out_host: torch.Tensor, stream=None) -> None:
        assert not x_host.is_cuda and not out_host.is_cuda and x_host.is_contiguous() and out_host.is_contiguous()
        _check(lib.ltxb_block_forward_host(self.handle, x_host.data_ptr(), out_host.data_ptr(), _stream(stream)))

    def join(self, stream=None) -> None:
        _check(lib.ltxb_host_pipe_join(self.handle, _stream(stream)))

    def free(self) -> None:
        if self.handle:
            lib.ltxb_host_pipe_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class QBlock(Block):
    """ltx/block.zig:481-611: the block with int8 g128 linears. Which linears
    are int8 is fixed when the weights are uploaded (the quant set)."""

    def qBlockOutAll(self, x, tstab, tidx, ctx, pts2, cos, sin):
        """ltx/block.zig:544-574: int8 q/k/v of both attentions and the FFN
        (weights uploaded with QSET_REF, or QSET_EXT which adds the output
        projections)."""
        if self.w.mode != MODE_INT8 or self.w.qset not in (QSET_REF, QSET_EXT):
            raise LtxbError(EINVAL, "qBlockOutAll needs int8 weights uploaded with QSET_REF or QSET_EXT")
        return self.forward(x, tstab, tidx, ctx, pts2, cos, sin)

    def qBlockOut(self, x, tstab, tidx, ctx, pts2, cos, sin):
        """ltx/block.zig:577-611: int8 q/k/v of both attentions, the FFN
        unquantised (weights uploaded with QSET_QKV)."""
        if self.w.mode != MODE_INT8 or self.w.qset != QSET_QKV:
            raise LtxbError(EINVAL, "qBlockOut needs int8 weights uploaded with QSET_QKV")
        return self.forward(x, tstab, tidx, ctx, pts2, cos, sin)


class Chain:
    """ltx/block.zig:434-455: three blocks (the harness's b0, b23, b47) run
    back to back on the same conditioning."""

    def __init__(self, b0: Block, b23: Block, b47: Block):
        self.b0, self.b23, self.b47 = b0, b23, b47

    def chainB23(self, x, tstab, tidx, ctx, pts2, cos, sin):
        y = self.b0.blockOut(x, tstab, tidx, ctx, pts2, cos, sin)
        return self.b23.blockOut(y, tstab, tidx, ctx, pts2, cos, sin)

    def chainB47(self, x, tstab, tidx, ctx, pts2, cos, sin):
        y = self.chainB23(x, tstab, tidx, ctx, pts2, cos, sin)
        return self.b47.blockOut(y, tstab, tidx, ctx, pts2, cos, sin)

    def wChainB47(self, x, tstab, tidx, ctx, pts2, cos, sin):
        """The same chain through wBlockOut (one function here: attention is
        always blockwise)."""
        y = self.b0.wBlockOut(x, tstab, tidx, ctx, pts2, cos, sin)
        y = self.b23.wBlockOut(y, tstab, tidx, ctx, pts2, cos, sin)
        return self.b47.wBlockOut(y, tstab, tidx, ctx, pts2, cos, sin)


# ---------------------------------------------------------------------------
# standalone operators
# ---------------------------------------------------------------------------

def attention(q, k, v, gate=None, scale: float | None = None, out=None, stream=None) -> torch.Tensor:
    """softmax(q k^T * scale) v per head; q [Tq, H, 128], k/v [Tkv, H, 128] bf16."""
    Tq, H, hd = q.shape
    assert hd == 128 and q.dtype == torch.bfloat16
    scale = 1.0 / np.sqrt(hd) if scale is None else scale
    out = torch.empty_like(q) if out is None else out
    _check(lib.ltxb_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(gate), Tq, k.shape[0], H, float(scale),
                              _stream(stream)))
    return out


def attention_split(q, k, v, gate=None, splits: int = 0, scale: float | None = None, out=None, workspace=None,
                    stream=None) -> torch.Tensor:
    """attention() computed as `splits` K/V ranges merged afterwards (0 = the
    library's choice for this GPU); for short query sequences."""
    Tq, H, hd = q.shape
    assert hd == 128 and q.dtype == torch.bfloat16
    scale = 1.0 / np.sqrt(hd) if scale is None else scale
    out = torch.empty_like(q) if out is None else out
    need = lib.ltxb_attention_split_workspace_bytes(Tq, k.shape[0], H, int(splits))
    if workspace is None:
        workspace = torch.empty(max(int(need), 1), dtype=torch.uint8, device=q.device)
    _check(lib.ltxb_attention_split(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(gate), Tq, k.shape[0], H,
                                    float(scale), int(splits), _ptr(workspace), workspace.numel(), _stream(stream)))
    return out


ROPE_LTX = 0
ROPE_AXES = 1


def rope_tables(kind: int, pos, n_heads: int, theta: float = 10000.0, stream=None):
    """cos, sin [T, H, 64] f32 on pos's device. ROPE_LTX: pos = grid [3, T, 2]
    (start, end) f32; ROPE_AXES: pos = [T, 3] (frame, row, col) f32."""
    pos = pos.contiguous().float()
    T = pos.shape[1] if kind == ROPE_LTX else pos.shape[0]
    cos = torch.empty(T, n_heads, 64, dtype=torch.float32, device=pos.device)
    sin = torch.empty_like(cos)
    _check(lib.ltxb_rope_tables(int(kind), _ptr(pos), T, n_heads, float(theta), _ptr(cos), _ptr(sin),
                                _stream(stream)))
    return cos, sin


def dq_gemm(a, wq, scales, bias=None, fused: bool = True, out=None, workspace=None, stream=None) -> torch.Tensor:
    """linQ: a [M, K] bf16 . dequant(wq [N, K] int8, scales [N, K/128])^T (+ bias) -> bf16 [M, N]."""
    M, K = a.shape
    N = wq.shape[0]
    sdt = DT_BF16 if scales.dtype == torch.bfloat16 else DT_F32
    out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device) if out is None else out
    if not fused and workspace is None:
        workspace = torch.empty(N * K * 2, dtype=torch.uint8, device=a.device)
    _check(lib.ltxb_dq_gemm(_ptr(a), _ptr(wq), _ptr(scales), sdt, _ptr(bias), _ptr(out), M, N, K, int(fused),
                            _ptr(workspace), 0 if workspace is None else workspace.numel(), _stream(stream)))
    return out


def stats_of(v, stream=None) -> tuple[float, float, float]:
    """statsOf (ltx/core_parts.zig:183-193) on the device: (NaN count, sum of
    squares, max |v|) of an f32 tensor, read back as three floats."""
    v = v.contiguous()
    out = torch.empty(3, dtype=torch.float32, device=v.device)
    ws = torch.empty(int(lib.ltxb_stats_workspace_bytes()), dtype=torch.uint8, device=v.device)
    _check(lib.ltxb_stats(_ptr(v), v.numel(), _ptr(out), _ptr(ws), ws.numel(), _stream(stream)))
    n, ss, ma = out.cpu().tolist()
    return n, ss, ma


def gemm_bf16(a, w, bias=None, out=None, stream=None) -> torch.Tensor:
    """lin on tcgen05: a [M, K] bf16 . w [N, K]^T (+ bias) -> bf16 [M, N]."""
    M, K = a.shape
    N = w.shape[0]
    out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device) if out is None else out
    _check(lib.ltxb_gemm_bf16(_ptr(a), _ptr(w), _ptr(bias), _ptr(out), M, N, K, _stream(stream)))
    return out
