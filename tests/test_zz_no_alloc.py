"""The no-allocation multihash entry point against the allocating one.

tcx_multihash_from_gpu_noalloc serves callers that cannot call cudaMalloc when they
need a content hash (an engine whose memory pool already holds nearly all of the GPU,
or a path that must not wait on cudaFree). It keeps its scratch in a fixed device
array inside the library. These checks call it through the C ABI and require the
same multihash as tcx_multihash_from_gpu, bit for bit, on two calls in a row (the
second call reuses the scratch the first one left behind). This file is named so
that pytest collects it last."""
import ctypes

import numpy as np
import pytest
import torch

from tensorcast_b200 import _native

pytestmark = pytest.mark.gpu


def _hash(fn_name, t: torch.Tensor, nbytes: int, leaf: int, stream=None):
    L = _native.lib()
    buf = ctypes.create_string_buffer(64)
    args = [t.data_ptr(), nbytes, t.device.index or 0, leaf, buf, 64]
    if fn_name.endswith("noalloc"):
        args.append(stream)
    rc = getattr(L, fn_name)(*args)
    return rc, (buf.value.decode() if rc == 0 else L.tcx_last_error().decode())


def test_noalloc_matches_allocating_entry_on_two_calls(cuda_device):
    rng = np.random.default_rng(2024)
    # First call: many leaves (level kernels + finish); second: fewer leaves, so any
    # stale scratch left by the first call would show up in the result.
    cases = [((96 << 20) + 12345, 8 << 10), ((5 << 20) + 7, 4 << 20)]
    for nbytes, leaf in cases:
        a = rng.integers(0, 256, size=nbytes, dtype=np.uint8)
        t = torch.from_numpy(a).cuda()
        torch.cuda.synchronize()
        rc_ref, want = _hash("tcx_multihash_from_gpu", t, nbytes, leaf)
        stream = torch.cuda.current_stream().cuda_stream
        rc, got = _hash("tcx_multihash_from_gpu_noalloc", t, nbytes, leaf, stream)
        assert rc_ref == 0 and rc == 0, (want, got)
        assert got == want


def test_noalloc_rejects_more_leaves_than_its_scratch(cuda_device):
    t = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    rc, msg = _hash("tcx_multihash_from_gpu_noalloc", t, 1 << 20, 64)  # 16384 leaves: fits
    assert rc == 0
    t2 = torch.zeros((1 << 20) + 64, dtype=torch.uint8, device="cuda")
    rc, msg = _hash("tcx_multihash_from_gpu_noalloc", t2, (1 << 20) + 64, 64)  # 16385 leaves
    assert rc == 3 and "no-alloc scratch capacity of 16384 leaves" in msg
