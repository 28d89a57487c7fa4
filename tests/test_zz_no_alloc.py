"""The no-allocation multihash entry point, checked against the CPU oracle.

tcx_multihash_from_gpu_noalloc serves callers that cannot call cudaMalloc when they
need a content hash: an inference engine whose memory pool already holds nearly all
of the GPU (a new allocation would fail or fragment that pool), or a latency-bound
path that must not wait on cudaFree, which synchronises the whole device. It keeps
its scratch in a fixed device array inside the library. These checks call it
through the C ABI:

* two calls in a row give the CPU oracle's multihash and the allocating entry
  point's, bit for bit (the second call reuses the scratch the first one left);
* a call leaves the device's free memory unchanged;
* in a fresh process whose device memory has been filled up, it still hashes a
  shape never hashed before in that process, while the allocating entry point
  fails for lack of memory;
* it rejects more leaves than its scratch holds and a stream of another device,
  and restores the caller's current device.

This file is named so that pytest collects it last."""
import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from oracle import oracle
from tensorcast_b200 import _native

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _hash(fn_name, ptr: int, nbytes: int, device: int, leaf: int, stream=None):
    L = _native.lib()
    buf = ctypes.create_string_buffer(64)
    args = [ctypes.c_void_p(ptr), nbytes, device, leaf, buf, 64]
    if fn_name.endswith("noalloc"):
        args.append(ctypes.c_void_p(stream))
    rc = getattr(L, fn_name)(*args)
    return rc, (buf.value.decode() if rc == 0 else L.tcx_last_error().decode())


def test_noalloc_matches_oracle_and_allocating_entry_on_two_calls(cuda_device):
    rng = np.random.default_rng(2024)
    # First call: many leaves (level kernels + finish); second: fewer leaves, so any
    # stale scratch left by the first call would show up in the result.
    cases = [((96 << 20) + 12345, 8 << 10), ((5 << 20) + 7, 4 << 20)]
    stream = torch.cuda.current_stream().cuda_stream
    for nbytes, leaf in cases:
        a = rng.integers(0, 256, size=nbytes, dtype=np.uint8)
        t = torch.from_numpy(a).cuda()
        torch.cuda.synchronize()
        rc, got = _hash("tcx_multihash_from_gpu_noalloc", t.data_ptr(), nbytes, 0, leaf, stream)
        assert rc == 0, got
        assert got == oracle.multihash_gpu_semantics(a, leaf)
        rc_ref, want = _hash("tcx_multihash_from_gpu", t.data_ptr(), nbytes, 0, leaf)
        assert rc_ref == 0, want
        assert got == want


def test_noalloc_leaves_free_memory_unchanged(cuda_device):
    a = np.random.default_rng(7).integers(0, 256, size=(33 << 20) + 3, dtype=np.uint8)
    t = torch.from_numpy(a).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    rc, first = _hash("tcx_multihash_from_gpu_noalloc", t.data_ptr(), a.size, 0, 16 << 10, stream)
    assert rc == 0, first
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    rc, second = _hash("tcx_multihash_from_gpu_noalloc", t.data_ptr(), a.size, 0, 16 << 10, stream)
    free1, _ = torch.cuda.mem_get_info()
    assert rc == 0 and second == first == oracle.multihash_gpu_semantics(a, 16 << 10)
    assert free1 == free0


_PRESSURE_CHILD = textwrap.dedent(r"""
    import ctypes, json, sys
    import numpy as np
    import torch
    sys.path.insert(0, sys.argv[1])
    from oracle import oracle
    from tensorcast_b200 import _native
    L = _native.lib()

    def call(fn, t, nbytes, leaf, stream=None):
        buf = ctypes.create_string_buffer(64)
        args = [ctypes.c_void_p(t.data_ptr()), nbytes, 0, leaf, buf, 64]
        if stream is not None:
            args.append(ctypes.c_void_p(stream))
        rc = getattr(L, fn)(*args)
        return rc, (buf.value.decode() if rc == 0 else L.tcx_last_error().decode())

    torch.cuda.set_device(0)
    rng = np.random.default_rng(11)
    warm = rng.integers(0, 256, size=(20 << 20) + 64, dtype=np.uint8)   # 5121 leaves of 4 KiB
    fresh = rng.integers(0, 256, size=(48 << 20) + 4000, dtype=np.uint8)  # 12289 leaves of 4 KiB
    big = np.zeros(64 << 20, dtype=np.uint8)                              # 1 Mi leaves of 64 B
    d_warm, d_fresh, d_big = (torch.from_numpy(x).cuda() for x in (warm, fresh, big))
    stream = torch.cuda.current_stream().cuda_stream
    # Set-up call (scratch address, kernels loaded) before memory runs out.
    rc, got = call("tcx_multihash_from_gpu_noalloc", d_warm, warm.size, 4096, stream)
    assert rc == 0 and got == oracle.multihash_gpu_semantics(warm, 4096), got
    torch.cuda.synchronize()
    hold, chunk = [], torch.cuda.mem_get_info()[0] - (64 << 20)
    while chunk >= (1 << 20):
        try:
            hold.append(torch.empty(chunk, dtype=torch.uint8, device="cuda"))
        except torch.OutOfMemoryError:
            chunk //= 2
    free_after_fill = torch.cuda.mem_get_info()[0]
    rc_a, msg_a = call("tcx_multihash_from_gpu", d_big, big.size, 64)
    out = {"free_after_fill": free_after_fill, "held": sum(h.numel() for h in hold), "alloc_rc": rc_a,
           "alloc_msg": msg_a, "free_before_noalloc": torch.cuda.mem_get_info()[0]}
    for k in range(2):
        rc, got = call("tcx_multihash_from_gpu_noalloc", d_fresh, fresh.size, 4096, stream)
        out[f"noalloc_rc{k}"], out[f"noalloc_ok{k}"] = rc, rc == 0 and got == oracle.multihash_gpu_semantics(fresh, 4096)
        out[f"noalloc_msg{k}"] = got
    out["free_end"] = torch.cuda.mem_get_info()[0]
    print(json.dumps(out))
""")


def test_noalloc_hashes_when_device_memory_is_full(cuda_device):
    """Fresh process: after a set-up call, fill the device's memory with tensors, then
    hash a shape never hashed in that process. The no-alloc entry point succeeds on two
    calls in a row (oracle multihash); the allocating one cannot get its buffers."""
    env = dict(os.environ, PYTORCH_CUDA_ALLOC_CONF="")
    proc = subprocess.run([sys.executable, "-c", _PRESSURE_CHILD, ROOT], capture_output=True, text=True, timeout=600,
                          env=env)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    import json
    out = json.loads(proc.stdout.strip().splitlines()[-1])
    assert out["free_after_fill"] < (64 << 20), out
    assert out["alloc_rc"] in (8, 13), out  # RESOURCE_EXHAUSTED or INTERNAL: its buffers could not be allocated
    assert out["noalloc_rc0"] == 0 and out["noalloc_ok0"], out
    assert out["noalloc_rc1"] == 0 and out["noalloc_ok1"], out
    assert out["free_end"] == out["free_before_noalloc"], out


def test_noalloc_rejects_more_leaves_than_its_scratch(cuda_device):
    t = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    rc, msg = _hash("tcx_multihash_from_gpu_noalloc", t.data_ptr(), 1 << 20, 0, 64)  # 16384 leaves: fits
    assert rc == 0, msg
    t2 = torch.zeros((1 << 20) + 64, dtype=torch.uint8, device="cuda")
    rc, msg = _hash("tcx_multihash_from_gpu_noalloc", t2.data_ptr(), (1 << 20) + 64, 0, 64)  # 16385 leaves
    assert rc == 3 and "no-alloc scratch capacity of 16384 leaves" in msg


def test_noalloc_checks_the_stream_device_and_restores_the_current_device(cuda_device):
    t = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    rc, msg = _hash("tcx_multihash_from_gpu_noalloc", t.data_ptr(), 1 << 20, 0, 1 << 16, s.cuda_stream)
    assert rc == 0, msg
    assert torch.cuda.current_device() == 0
    if torch.cuda.device_count() > 1:
        # A stream of device 1 with device_id 0 is rejected; the current device stays 1.
        with torch.cuda.device(1):
            s1 = torch.cuda.Stream()
            rc, msg = _hash("tcx_multihash_from_gpu_noalloc", t.data_ptr(), 1 << 20, 0, 1 << 16, s1.cuda_stream)
            assert rc == 3 and "belongs to device 1" in msg, msg
            rc, msg = _hash("tcx_multihash_from_gpu_noalloc", t.data_ptr(), 1 << 20, 0, 1 << 16, None)
            assert rc == 0, msg
            assert torch.cuda.current_device() == 1
