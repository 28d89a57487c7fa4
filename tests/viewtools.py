"""Test helpers: random artifacts, per-rank view specs, and a numpy executor of the
native exchange schedule (tcx_plan_exchange) so the host planning can be checked on CPU."""
from __future__ import annotations

import numpy as np

from tensorcast_b200.artifact import CanonicalEntry, CanonicalIndex, compact_stride
from tensorcast_b200.views import ViewSpec, NarrowOp, TransposeOp, plan_view

UINT = {1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}
DT = {1: "torch.uint8", 2: "torch.bfloat16", 4: "torch.float32", 8: "torch.int64"}


def random_tensors(seed: int, n: int = 12, odd: bool = True) -> dict:
    """name -> (raw uint8 bytes, shape, esize); odd sizes exercise the 8-byte pads."""
    rng = np.random.default_rng(seed)
    out = {}
    for i in range(n):
        es = int(rng.choice([1, 2, 4, 8])) if odd else 2
        nd = int(rng.integers(1, 4))
        shape = tuple(int(x) for x in rng.integers(1, 9, size=nd) * (1 if odd else 8))
        if nd >= 2 and rng.random() < 0.5:
            shape = (shape[0] * 4,) + shape[1:]
        numel = int(np.prod(shape))
        raw = rng.integers(0, 256, size=numel * es, dtype=np.uint8)
        out[f"t{i:02d}.{rng.integers(0, 99)}"] = (raw, shape, es)
    return out


def index_from_meta(meta: dict, total: int) -> CanonicalIndex:
    entries = {}
    for name in sorted(meta, key=lambda s: s.encode("utf-8")):
        off, shape, es = meta[name]
        entries[name] = CanonicalEntry(off, int(np.prod(shape)) * es if shape else es, tuple(shape),
                                       compact_stride(shape), DT[es], 0)
    return CanonicalIndex(entries, total, {})


def random_view(meta: dict, rng, allow_fused=False):
    """A random (slices, transpose, subset) triple in oracle form, and the ViewSpec."""
    slices, transpose, spec = {}, {}, ViewSpec()
    for name, (_, shape, _) in meta.items():
        r = rng.random()
        if r < 0.4:
            d = int(rng.integers(0, len(shape)))
            ext = shape[d]
            s = int(rng.integers(0, ext))
            ln = int(rng.integers(1, ext - s + 1))
            if not (s == 0 and ln == ext):
                slices[name] = (d, s, ln)
                spec.tensors.setdefault(name, []).append(NarrowOp(d, s, ln))
        elif r < 0.6 and len(shape) >= 2:
            a, b = rng.choice(len(shape), 2, replace=False)
            transpose[name] = [(int(a), int(b))]
            spec.tensors.setdefault(name, []).append(TransposeOp(int(a), int(b)))
    subset = None
    if rng.random() < 0.5:
        names = list(meta)
        k = int(rng.integers(1, len(names) + 1))
        subset = [names[i] for i in rng.permutation(len(names))[:k]]
        if rng.random() < 0.3:
            subset = subset + subset[:1]  # duplicates keep the first occurrence
    return slices, transpose, subset, spec


def apply_jobs(src: np.ndarray, dst: np.ndarray, jobs: np.ndarray) -> None:
    for j in jobs:
        so, do, sp, dp, rb, rows = (int(j[k]) for k in ("src_off", "dst_off", "src_pitch", "dst_pitch",
                                                          "row_bytes", "rows"))
        for k in range(rows):
            dst[do + k * dp: do + k * dp + rb] = src[so + k * sp: so + k * sp + rb]


def apply_permutes(view: np.ndarray, permutes: list) -> None:
    for p in permutes:
        shape, es = p["shape"], p["esize"]
        n = int(np.prod(shape)) * es
        a = view[p["dst_off"]: p["dst_off"] + n].view(UINT[es]).reshape(shape)
        view[p["dst_off"]: p["dst_off"] + n] = np.ascontiguousarray(np.transpose(a, p["perm"])).view(np.uint8).reshape(-1)


def emulate_load(canon: np.ndarray, bounds, rank_plans, exch: list) -> list:
    """Runs every rank's exchange schedule in numpy; returns each rank's view bytes."""
    world = len(bounds) - 1
    sends = []
    views = []
    for r in range(world):
        stage = canon[bounds[r]:bounds[r + 1]]
        x = exch[r]
        send = np.zeros(int(x["send_offsets"][-1]), np.uint8)
        apply_jobs(stage, send, x["pack"])
        sends.append(send)
        view = np.full(rank_plans[r].view_bytes, 0xA5, np.uint8)
        for off, ln in x["gaps"]:
            view[int(off): int(off) + int(ln)] = 0
        apply_jobs(stage, view, x["local"])
        views.append(view)
    for r in range(world):
        x = exch[r]
        recv = np.zeros(int(x["recv_offsets"][-1]), np.uint8)
        for p in range(world):
            if p == r:
                continue
            xp = exch[p]
            data = sends[p][int(xp["send_offsets"][r]): int(xp["send_offsets"][r + 1])]
            assert data.size == int(x["recv_counts"][p]), (r, p, data.size, x["recv_counts"][p])
            if x["direct"][p]:
                o = int(x["recv_view_off"][p])
                views[r][o: o + data.size] = data
            else:
                o = int(x["recv_offsets"][p])
                assert int(x["recv_offsets"][p + 1]) - o == data.size
                recv[o: o + data.size] = data
        apply_jobs(recv, views[r], x["scatter"])
        apply_permutes(views[r], rank_plans[r].permutes)
    return views
