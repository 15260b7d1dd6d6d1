"""CPU tests of the streaming staging ring (ltxb_stage_*, the B200 form of
ltx/loader.zig:176-321): the schedule check before any I/O, in-order staging
through two host slots by the reader thread, the digest check on first
touch, bounded waits, abort, and the slot state machine. Plain host memory
(pinned=False) so no GPU is needed; the device upload from a slot is the
GPU test's part."""

import numpy as np
import pytest

import ltxb
from ltxb import blobfmt


def _blob_dirs(tmp_path, sizes, seed=0):
    rng = np.random.default_rng(seed)
    dirs = []
    for i, n in enumerate(sizes):
        tensors = [(f"transformer_blocks.{i}.t{j}", "F32", [n // 4],
                    rng.standard_normal(n // 4).astype(np.float32).tobytes()) for j in range(3)]
        d = tmp_path / f"block{i}"
        blobfmt.write_dir(d, tensors, block=i)
        dirs.append(d)
    return dirs


def _open_all(dirs, verify_digest=False):
    return [ltxb.Blob.open(d, verify_digest=verify_digest) for d in dirs]


def test_stage_streams_the_schedule_in_order(tmp_path):
    dirs = _blob_dirs(tmp_path, [4096, 12288, 1000])
    blobs = _open_all(dirs)
    schedule = [0, 1, 2, 1, 0, 2, 2, 1]
    st = ltxb.Stage(blobs, schedule, pinned=False, verify=True)
    try:
        for pos, bi in enumerate(schedule):
            got = st.acquire(pos, timeout_ms=10000)
            assert bytes(got) == (dirs[bi] / "blob.bin").read_bytes(), pos
            st.release(pos)
        s = st.stats()
        assert s["staged_bytes"] == sum(len(blobs[i].data) for i in schedule)
        assert s["verify_ns"] > 0 and s["copy_ns"] > 0
    finally:
        st.free()


def test_stage_holds_two_positions_at_once(tmp_path):
    """Both slots can be in use together; a third position then waits (and
    times out) until one of them is released."""
    dirs = _blob_dirs(tmp_path, [2048, 2048, 2048], seed=1)
    blobs = _open_all(dirs)
    st = ltxb.Stage(blobs, [0, 1, 2], pinned=False, verify=False)
    try:
        a = st.acquire(0)
        b = st.acquire(1)
        assert bytes(a) == (dirs[0] / "blob.bin").read_bytes() and bytes(b) == (dirs[1] / "blob.bin").read_bytes()
        with pytest.raises(ltxb.LtxbError) as ei:
            st.acquire(2, timeout_ms=200)
        assert ei.value.code == ltxb.ETIMEOUT
        st.release(0)
        assert bytes(st.acquire(2, timeout_ms=10000)) == (dirs[2] / "blob.bin").read_bytes()
        st.release(1)
        st.release(2)
    finally:
        st.free()


def test_stage_schedule_checked_before_io(tmp_path):
    dirs = _blob_dirs(tmp_path, [4096, 8192], seed=2)
    blobs = _open_all(dirs)
    with pytest.raises(ltxb.LtxbError, match="ScheduleOutOfRange"):
        ltxb.Stage(blobs, [0, 2], pinned=False)
    with pytest.raises(ltxb.LtxbError, match="ScheduleOutOfRange"):
        ltxb.Stage(blobs, [-1], pinned=False)
    with pytest.raises(ltxb.LtxbError, match="SlotTooSmall"):
        ltxb.Stage(blobs, [0, 1], slot_bytes=len(blobs[0].data), pinned=False)


def test_stage_digest_checked_on_first_touch(tmp_path):
    """A blob whose bytes do not hash to the manifest's digest fails when the
    reader first stages it; the consumer gets the reader's error."""
    dirs = _blob_dirs(tmp_path, [4096, 4096], seed=3)
    data = bytearray((dirs[1] / "blob.bin").read_bytes())
    data[17] ^= 1
    (dirs[1] / "blob.bin").write_bytes(bytes(data))
    blobs = _open_all(dirs)  # no digest check at open
    st = ltxb.Stage(blobs, [0, 1], pinned=False, verify=True)
    try:
        st.acquire(0)
        st.release(0)
        with pytest.raises(ltxb.LtxbError, match="BlobDigestMismatch"):
            st.acquire(1, timeout_ms=10000)
    finally:
        st.free()


def test_stage_abort_and_state_machine(tmp_path):
    dirs = _blob_dirs(tmp_path, [1024, 1024, 1024], seed=4)
    blobs = _open_all(dirs)
    st = ltxb.Stage(blobs, [0, 1, 2, 0], pinned=False, verify=False)
    try:
        st.acquire(0)
        with pytest.raises(ltxb.LtxbError):  # a position that is not held
            st.release(1)
        st.release(0)
        with pytest.raises(ltxb.LtxbError):  # released twice
            st.release(0)
        with pytest.raises(ltxb.LtxbError):  # outside the schedule
            st.acquire(4)
        st.abort()
        with pytest.raises(ltxb.LtxbError, match="RingShutdown"):
            st.acquire(1, timeout_ms=1000)
    finally:
        st.free()  # joins the reader even though it was parked or aborted


def test_stage_free_while_reader_waits(tmp_path):
    """Freeing the stage with both slots full and the reader parked on a free
    slot ends the reader (no deadlock at teardown)."""
    dirs = _blob_dirs(tmp_path, [1024, 1024, 1024], seed=5)
    blobs = _open_all(dirs)
    st = ltxb.Stage(blobs, [0, 1, 2, 1, 0], pinned=False, verify=False)
    st.acquire(0)
    st.acquire(1)
    st.free()
