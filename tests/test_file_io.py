"""Host staging reads (tcx_read_segments_ex): source-ordered preads, O_DIRECT windows with
unaligned segments, the buffered fallback where O_DIRECT is refused, short reads."""
import os

import numpy as np
import pytest

from tensorcast_b200 import _native
from tensorcast_b200.loader import read_segments


def _segments(rng, file_size, n, max_len):
    """Random unaligned (file_offset, length) ranges placed back to back in a destination,
    listed in a shuffled order (not the file order)."""
    segs, cursor = [], 0
    for _ in range(n):
        ln = int(rng.integers(1, max_len))
        off = int(rng.integers(0, file_size - ln))
        segs.append((off, cursor, ln))
        cursor += ln
    order = rng.permutation(len(segs))
    return [segs[i] for i in order], cursor


@pytest.mark.parametrize("direct", [False, True])
def test_read_segments_unaligned_any_order(tmp_path, direct):
    rng = np.random.default_rng(5)
    data = rng.integers(0, 256, (40 << 20) + 1234, dtype=np.uint8)
    a, b = tmp_path / "a.bin", tmp_path / "b.bin"
    data.tofile(a)
    data[::-1].copy().tofile(b)
    segs, total = _segments(rng, data.size, 60, 300_000)
    segs += [(123, total, (20 << 20) + 77)]  # one segment longer than a direct window
    total += (20 << 20) + 77
    out = np.zeros(total, np.uint8)
    want = np.zeros(total, np.uint8)
    listed = []
    for i, (off, dst, ln) in enumerate(segs):
        path, src = (a, data) if i % 3 else (b, data[::-1])
        listed.append((str(path), off, dst, ln))
        want[dst:dst + ln] = src[off:off + ln]
    read_segments(listed, out.ctypes.data, threads=4, direct=direct)
    assert (out == want).all()


def test_read_segments_direct_falls_back_on_tmpfs():
    if not os.path.isdir("/dev/shm"):
        pytest.skip("no /dev/shm")
    p = f"/dev/shm/tcx_file_io_{os.getpid()}.bin"
    data = np.random.default_rng(1).integers(0, 256, 1 << 20, dtype=np.uint8)
    data.tofile(p)
    try:
        out = np.zeros(5000, np.uint8)
        read_segments([(p, 4097, 0, 3000), (p, 17, 3000, 2000)], out.ctypes.data, threads=2, direct=True)
        assert (out[:3000] == data[4097:7097]).all() and (out[3000:] == data[17:2017]).all()
    finally:
        os.unlink(p)


@pytest.mark.parametrize("direct", [False, True])
def test_read_segments_short_read_is_data_loss(tmp_path, direct):
    p = tmp_path / "short.bin"
    p.write_bytes(b"x" * 10000)
    out = np.zeros(8192, np.uint8)
    with pytest.raises(_native.TcxError, match="short read") as ei:
        read_segments([(str(p), 5000, 0, 8000)], out.ctypes.data, threads=1, direct=direct)
    assert ei.value.code == 15
    with pytest.raises(_native.TcxError, match="open failed") as ei:
        read_segments([(str(tmp_path / "missing.bin"), 0, 0, 10)], out.ctypes.data, threads=1, direct=direct)
    assert ei.value.code == 5
