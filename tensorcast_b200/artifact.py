"""Safetensors sources and the canonical byte space.

Mirrors the reference's metadata layer:

* ``parse_safetensors_header``      -> ParseSafetensorsHeader (safetensors_util.h:15-40)
* ``SAFETENSORS_DTYPES``            -> dtype map (safetensors_util.cc:67-78) and element
                                        sizes (view_planner.cc:113-135)
* ``build_canonical_index``         -> build_coalesced_canonical_index_from_source_index_json
                                        (canonical_index.cc:155-221): names sorted bytewise,
                                        every tensor start aligned to 8 bytes
* ``canonical_index_json``          -> build_canonical_index_json (canonical_index.cc:120-152):
                                        {"name":[offset,size,shape,stride,dtype,storage_offset]}
* ``canonical_segments``            -> the file reads that assemble a range of the canonical
                                        byte space (MultiSafetensorsSource, multi_safetensors_source.h:21-58)
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass, field

# safetensors dtype -> (torch dtype string, element size)
SAFETENSORS_DTYPES = {
    "BF16": ("torch.bfloat16", 2),
    "F16": ("torch.float16", 2),
    "F32": ("torch.float32", 4),
    "F64": ("torch.float64", 8),
    "I8": ("torch.int8", 1),
    "U8": ("torch.uint8", 1),
    "I16": ("torch.int16", 2),
    "I32": ("torch.int32", 4),
    "I64": ("torch.int64", 8),
    "BOOL": ("torch.bool", 1),
    "F8_E4M3": ("torch.float8_e4m3fn", 1),
    "F8_E5M2": ("torch.float8_e5m2", 1),
}
ELEMENT_SIZE = {v[0]: v[1] for v in SAFETENSORS_DTYPES.values()}
ELEMENT_SIZE.update({"torch.float": 4, "torch.double": 8})
CANONICAL_ALIGN = 8


@dataclass(frozen=True)
class SourceTensor:
    name: str
    path: str
    file_offset: int  # absolute byte offset of the tensor in its file
    nbytes: int
    shape: tuple
    dtype: str  # torch dtype string

    @property
    def esize(self) -> int:
        return ELEMENT_SIZE[self.dtype]


@dataclass(frozen=True)
class CanonicalEntry:
    offset: int
    size: int
    shape: tuple
    stride: tuple
    dtype: str
    storage_offset: int = 0

    @property
    def esize(self) -> int:
        return ELEMENT_SIZE[self.dtype]


def compact_stride(shape) -> tuple:
    stride, acc = [], 1
    for d in reversed(shape):
        stride.append(acc)
        acc *= int(d)
    return tuple(reversed(stride))


def parse_safetensors_header(path: str) -> tuple[int, dict]:
    """Returns (payload offset, header dict without __metadata__)."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header)")
        (n,) = struct.unpack("<Q", head)
        if n > (100 << 20):
            raise ValueError(f"{path}: safetensors header too large ({n} bytes)")
        raw = f.read(n)
    if len(raw) != n:
        raise ValueError(f"{path}: truncated safetensors header")
    hdr = json.loads(raw)
    hdr.pop("__metadata__", None)
    return 8 + n, hdr


def build_source_index(paths) -> dict[str, SourceTensor]:
    """Tensors of one or more safetensors files (names must be unique across files)."""
    if isinstance(paths, (str, os.PathLike)):
        paths = [paths]
    out: dict[str, SourceTensor] = {}
    for p in paths:
        p = os.fspath(p)
        base, hdr = parse_safetensors_header(p)
        size = os.path.getsize(p)
        for name, meta in hdr.items():
            dt = meta["dtype"]
            if dt not in SAFETENSORS_DTYPES:
                raise ValueError(f"unsupported safetensors dtype {dt} for tensor {name}")
            tdt, es = SAFETENSORS_DTYPES[dt]
            b, e = meta["data_offsets"]
            shape = tuple(int(x) for x in meta["shape"])
            numel = 1
            for d in shape:
                numel *= d
            if e - b != numel * es:
                raise ValueError(f"tensor {name}: data_offsets span {e - b} bytes, shape needs {numel * es}")
            if base + e > size:
                raise ValueError(f"tensor {name} extends past the end of {p}")
            if name in out:
                raise ValueError(f"duplicate tensor name {name} across safetensors files")
            out[name] = SourceTensor(name, p, base + b, e - b, shape, tdt)
    return out


def safetensors_files(path: str) -> list[str]:
    """A file, or every *.safetensors file of a directory (sorted)."""
    if os.path.isdir(path):
        files = sorted(os.path.join(path, f) for f in os.listdir(path) if f.endswith(".safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {path}")
        return files
    return [path]


@dataclass
class CanonicalIndex:
    entries: dict  # name -> CanonicalEntry, in canonical (sorted) order
    total_bytes: int
    sources: dict = field(default_factory=dict)  # name -> SourceTensor

    def names(self) -> list[str]:
        return list(self.entries)

    def to_json(self) -> str:
        return canonical_index_json(self.entries)


def build_canonical_index(sources: dict[str, SourceTensor], align: int = CANONICAL_ALIGN) -> CanonicalIndex:
    if align <= 0:
        raise ValueError("align_bytes must be > 0")
    entries: dict[str, CanonicalEntry] = {}
    cursor = 0
    for name in sorted(sources, key=lambda s: s.encode("utf-8")):
        st = sources[name]
        if cursor % align:
            cursor += align - cursor % align
        entries[name] = CanonicalEntry(cursor, st.nbytes, st.shape, compact_stride(st.shape), st.dtype, 0)
        cursor += st.nbytes
    return CanonicalIndex(entries, cursor, dict(sources))


def canonical_index_json(entries: dict) -> str:
    obj = {name: [e.offset, e.size, list(e.shape), list(e.stride), e.dtype, e.storage_offset]
           for name, e in sorted(entries.items(), key=lambda kv: kv[0].encode("utf-8"))}
    return json.dumps(obj, separators=(",", ":"))


def canonical_segments(index: CanonicalIndex, lo: int, hi: int) -> list[tuple[str, int, int, int]]:
    """File reads (path, file_offset, dst_offset relative to lo, length) covering the tensor
    bytes of canonical range [lo, hi); pad bytes between tensors are not covered."""
    segs = []
    for name, e in index.entries.items():
        a, b = max(lo, e.offset), min(hi, e.offset + e.size)
        if a >= b:
            continue
        st = index.sources[name]
        segs.append((st.path, st.file_offset + (a - e.offset), a - lo, b - a))
    return merge_segments(segs)


def merge_segments(segs):
    out = []
    for s in segs:
        if out and out[-1][0] == s[0] and out[-1][1] + out[-1][3] == s[1] and out[-1][2] + out[-1][3] == s[2]:
            p = out[-1]
            out[-1] = (p[0], p[1], p[2], p[3] + s[3])
        else:
            out.append(s)
    return out


def pad_ranges(index: CanonicalIndex, lo: int, hi: int) -> list[tuple[int, int]]:
    """(offset relative to lo, length) of canonical bytes in [lo, hi) that no tensor covers."""
    out, cursor = [], lo
    for e in index.entries.values():
        a, b = max(lo, e.offset), min(hi, e.offset + e.size)
        if a >= b:
            continue
        if a > cursor:
            out.append((cursor - lo, a - cursor))
        cursor = max(cursor, b)
    if hi > cursor:
        out.append((cursor - lo, hi - cursor))
    return out
