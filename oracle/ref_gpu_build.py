"""Builds the reference's own GPU SHA-256 kernel for B200 timing. TEST/BENCH INFRASTRUCTURE ONLY.

The reference compiles its only GPU kernel at run time: the CUDA source is a raw
string (kSha256KernelSource) inside core/common/artifact_hash_gpu.cc:193-412, given
to NVRTC as "tensorcast_sha256.cu" with the options "--std=c++17" and
"--gpu-architecture=compute_<major><minor>" of the current device (:505-516), and
the resulting PTX is loaded through the driver (JIT to the device's SASS). This
script does the same from the source where it lies under the reference tree:

    python oracle/ref_gpu_build.py [REFERENCE_ROOT]

writes oracle/_ref/tensorcast_sha256_compute_100.ptx (compute_100 = B200, CC 10.0)
with this container's NVRTC. The text is read from the reference file at build
time and never copied into the repository; oracle/_ref/ is git-ignored (but travels
to the GPU box with the built launcher, oracle/_ref/libref_gpu.so, see
oracle/ref_gpu_launch.cc and oracle/Makefile). Nothing in tensorcast_b200/ uses
either file: bench.py times the reference kernel beside the product kernel.
"""
from __future__ import annotations

import ctypes
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
SOURCE_REL = os.path.join("core", "common", "artifact_hash_gpu.cc")
BEGIN, END = 'kSha256KernelSource[] = R"NVRTC(', ')NVRTC";'
ARCH = "compute_100"


def extract(ref_root: str) -> str:
    with open(os.path.join(ref_root, SOURCE_REL), encoding="utf-8") as f:
        text = f.read()
    i = text.index(BEGIN) + len(BEGIN)
    j = text.index(END, i)
    return text[i:j]


def nvrtc_compile(src: str, name: str, options: list[str]) -> bytes:
    cand = [os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "lib64", "libnvrtc.so"), "libnvrtc.so.12",
            "libnvrtc.so"]
    lib = None
    for c in cand:
        try:
            lib = ctypes.CDLL(c)
            break
        except OSError:
            continue
    if lib is None:
        raise SystemExit("libnvrtc not found")
    prog = ctypes.c_void_p()
    rc = lib.nvrtcCreateProgram(ctypes.byref(prog), src.encode(), name.encode(), 0, None, None)
    if rc:
        raise SystemExit(f"nvrtcCreateProgram failed: {rc}")
    opts = (ctypes.c_char_p * len(options))(*[o.encode() for o in options])
    rc = lib.nvrtcCompileProgram(prog, len(options), opts)
    log_size = ctypes.c_size_t()
    lib.nvrtcGetProgramLogSize(prog, ctypes.byref(log_size))
    log = ctypes.create_string_buffer(max(log_size.value, 1))
    lib.nvrtcGetProgramLog(prog, log)
    if rc:
        raise SystemExit(f"nvrtcCompileProgram failed ({rc}): {log.value.decode(errors='replace')}")
    size = ctypes.c_size_t()
    lib.nvrtcGetPTXSize(prog, ctypes.byref(size))
    ptx = ctypes.create_string_buffer(size.value)
    lib.nvrtcGetPTX(prog, ptx)
    lib.nvrtcDestroyProgram(ctypes.byref(prog))
    return ptx.raw.rstrip(b"\0")


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else "/root/reference"
    if not os.path.exists(os.path.join(ref_root, SOURCE_REL)):
        raise SystemExit(f"reference source not found under {ref_root}")
    ptx = nvrtc_compile(extract(ref_root), "tensorcast_sha256.cu", ["--std=c++17", f"--gpu-architecture={ARCH}"])
    os.makedirs(OUT_DIR, exist_ok=True)
    out = os.path.join(OUT_DIR, f"tensorcast_sha256_{ARCH}.ptx")
    with open(out + ".tmp", "wb") as f:
        f.write(ptx)
    os.replace(out + ".tmp", out)
    print(out)


if __name__ == "__main__":
    main()
