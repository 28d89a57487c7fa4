"""bind_into: loads straight into caller-owned tensors (tensorcast_b200.binding, api.bind_into).

CPU tests restate the reference's copy-plan tests (tests/python/api/test_mapped_binding.py:
JSON round trip with the exact encoding, normalisation of dicts and tuples, target-name and
gap checks) and check the copy jobs by applying them in numpy. GPU tests load through
tcx_group_load (TCX_LOAD_TARGETS) and compare every target with safetensors' own reader."""
import os

import numpy as np
import pytest
import torch

from tensorcast_b200 import api
from tensorcast_b200.artifact import build_canonical_index, build_source_index
from tensorcast_b200.binding import (CopyPlanEntry, Range, copy_plan_from_json, copy_plan_to_json, mapped_copy_jobs,
                                     normalize_copy_plan, validate_copy_plan)
from tensorcast_b200.synthetic import llama_shapes, tiny_llama, write_safetensors


class _Index:
    """A canonical index over one uint8 tensor 'src' of 8 bytes (the reference tests' index)."""

    def __init__(self):
        from tensorcast_b200.artifact import CanonicalEntry
        self.entries = {"src": CanonicalEntry(0, 8, (8,), (1,), "torch.uint8", 0)}


def test_copy_plan_json_roundtrip():
    plan = [CopyPlanEntry("src", Range(0, 0, 4), "a", Range(0, 0, 4)),
            CopyPlanEntry("src", Range(0, 4, 8), "b", Range(0, 0, 4))]
    enc = copy_plan_to_json(plan)
    assert enc == ('{"entries":[{"ckpt_name":"src","ckpt_range":{"dim":0,"end":4,"start":0},"dst_name":"a",'
                   '"dst_range":{"dim":0,"end":4,"start":0}},{"ckpt_name":"src","ckpt_range":{"dim":0,"end":8,'
                   '"start":4},"dst_name":"b","dst_range":{"dim":0,"end":4,"start":0}}],"version":1}')
    assert copy_plan_from_json(enc) == tuple(plan)
    with pytest.raises(api.ArtifactError, match="Unsupported copy plan version"):
        copy_plan_from_json('{"version":2,"entries":[]}')


def test_normalize_copy_plan_accepts_dicts_and_tuples():
    plan = normalize_copy_plan([
        {"ckpt_name": "src", "ckpt_range": {"dim": 0, "start": 0, "end": 4}, "dst_name": "a",
         "dst_range": {"dim": 0, "start": 0, "end": 4}},
        ("src", {"dim": 0, "start": 4, "end": 8}, "b", {"dim": 0, "start": 0, "end": 4})])
    assert plan == (CopyPlanEntry("src", Range(0, 0, 4), "a", Range(0, 0, 4)),
                    CopyPlanEntry("src", Range(0, 4, 8), "b", Range(0, 0, 4)))
    with pytest.raises(api.ArtifactError, match="non-empty sequence"):
        normalize_copy_plan([])


def test_validate_copy_plan_names_and_gaps():
    idx = _Index()
    with pytest.raises(api.ArtifactError) as ei:
        validate_copy_plan(plan=[CopyPlanEntry("src", Range(0, 0, 4), "b", Range(0, 0, 4))], canonical_index=idx,
                           target_tensors={"a": torch.empty(4, dtype=torch.uint8)})
    assert ei.value.status_code == "FAILED_PRECONDITION"
    with pytest.raises(api.ArtifactError, match="has gaps before entry") as ei:
        validate_copy_plan(plan=[CopyPlanEntry("src", Range(0, 0, 3), "a", Range(0, 1, 4)),
                                 CopyPlanEntry("src", Range(0, 4, 8), "b", Range(0, 0, 4))], canonical_index=idx,
                           target_tensors={"a": torch.empty(4, dtype=torch.uint8),
                                           "b": torch.empty(4, dtype=torch.uint8)})
    assert ei.value.status_code == "INVALID_ARGUMENT"
    with pytest.raises(api.ArtifactError, match="element count mismatch"):
        validate_copy_plan(plan=[CopyPlanEntry("src", Range(0, 0, 3), "a", Range(0, 0, 4))], canonical_index=idx,
                           target_tensors={"a": torch.empty(4, dtype=torch.uint8)})
    with pytest.raises(api.ArtifactError, match="dtype mismatch"):
        validate_copy_plan(plan=[CopyPlanEntry("src", Range(0, 0, 4), "a", None)], canonical_index=idx,
                           target_tensors={"a": torch.empty(2, dtype=torch.int16)})
    with pytest.raises(api.ArtifactError, match="range outside view bounds"):
        validate_copy_plan(plan=[CopyPlanEntry("src", Range(0, 0, 4), "a", None)], canonical_index=idx,
                           target_tensors={"a": torch.empty(4, dtype=torch.uint8)}, view_narrows={"src": Range(0, 2, 8)})


def _apply(jobs, src: np.ndarray, mem: np.ndarray) -> None:
    for j in jobs:
        for r in range(int(j["rows"])):
            s = int(j["src_off"]) + r * int(j["src_pitch"])
            d = int(j["dst_off"]) + r * int(j["dst_pitch"])
            mem[d:d + int(j["row_bytes"])] = src[s:s + int(j["row_bytes"])]


def test_mapped_copy_jobs_concat_and_rect2d(tmp_path):
    """Fused QKV (concat on dim 0) and o_proj split into column halves (dim-1 rect2d),
    applied in numpy to targets carved out of one host buffer."""
    path = tmp_path / "m.safetensors"
    write_safetensors(str(path), llama_shapes(tiny_llama(layers=1, hidden=64, heads=4, kv_heads=2, head_dim=16)), 3,
                      device="cpu")
    index = build_canonical_index(build_source_index([str(path)]))
    from safetensors.torch import load_file
    ref = load_file(str(path))
    canon = np.zeros(index.total_bytes, np.uint8)
    for n, e in index.entries.items():
        canon[e.offset:e.offset + e.size] = ref[n].contiguous().view(torch.uint8).reshape(-1).numpy()
    p = "model.layers.0.self_attn."
    mem = torch.zeros(1 << 16, dtype=torch.uint8)
    qkv = mem[0:(64 + 32 + 32) * 64 * 2].view(torch.bfloat16).view(128, 64)
    o_lo = mem[20000:20000 + 64 * 32 * 2].view(torch.bfloat16).view(64, 32)
    o_hi = mem[30000:30000 + 64 * 32 * 2].view(torch.bfloat16).view(64, 32)
    targets = {"qkv": qkv, "o_lo": o_lo, "o_hi": o_hi}
    plan = [CopyPlanEntry(p + "q_proj.weight", None, "qkv", Range(0, 0, 64)),
            CopyPlanEntry(p + "k_proj.weight", None, "qkv", Range(0, 64, 96)),
            CopyPlanEntry(p + "v_proj.weight", None, "qkv", Range(0, 96, 128)),
            CopyPlanEntry(p + "o_proj.weight", Range(1, 0, 32), "o_lo", None),
            CopyPlanEntry(p + "o_proj.weight", Range(1, 32, 64), "o_hi", None)]
    # validation wants whole tensors (storage_offset 0, as the reference's); the jobs are
    # computed for targets carved out of one buffer so numpy can apply them
    validate_copy_plan(plan=plan, canonical_index=index,
                       target_tensors={k: torch.empty_like(v) for k, v in targets.items()})
    jobs = mapped_copy_jobs(plan, index, targets, mem.data_ptr())
    assert int(jobs[3]["rows"]) == 64 and int(jobs[3]["dst_pitch"]) == 64 and int(jobs[3]["src_pitch"]) == 128
    m = mem.numpy()
    _apply(jobs, canon, m)
    assert torch.equal(qkv, torch.cat([ref[p + "q_proj.weight"], ref[p + "k_proj.weight"], ref[p + "v_proj.weight"]]))
    assert torch.equal(o_lo, ref[p + "o_proj.weight"][:, :32]) and torch.equal(o_hi, ref[p + "o_proj.weight"][:, 32:])


@pytest.fixture(scope="module")
def artifact(tmp_path_factory):
    d = tmp_path_factory.mktemp("bind")
    path = os.path.join(d, "model.safetensors")
    write_safetensors(path, llama_shapes(tiny_llama(layers=2, hidden=128, heads=4, kv_heads=2, head_dim=32, ffn=256,
                                                    vocab=512)), 6, device="cpu")
    return path


@pytest.mark.gpu
def test_bind_into_view_tensors(cuda_device, artifact):
    from safetensors.torch import load_file
    ref = load_file(artifact)
    names = ["lm_head.weight", "model.layers.0.mlp.down_proj.weight", "model.norm.weight",
             "model.layers.1.self_attn.o_proj.weight"]
    art = api.from_disk(artifact).subset(names).view(
        slices={"lm_head.weight": slice(128, 256), "model.layers.0.mlp.down_proj.weight": (1, slice(64, 192))},
        transpose={"model.layers.1.self_attn.o_proj.weight": [(0, 1)]})
    want = {"lm_head.weight": ref["lm_head.weight"][128:256],
            "model.layers.0.mlp.down_proj.weight": ref["model.layers.0.mlp.down_proj.weight"][:, 64:192],
            "model.norm.weight": ref["model.norm.weight"],
            "model.layers.1.self_attn.o_proj.weight": ref["model.layers.1.self_attn.o_proj.weight"].t()}
    # separate allocations in reverse order, with guard bytes around each
    guards, targets = [], {}
    for n in reversed(names):
        g = torch.full((want[n].numel() * 2 + 512,), 0xA5, dtype=torch.uint8, device="cuda")
        guards.append(g)
        targets[n] = g[256:256 + want[n].numel() * 2].view(torch.bfloat16).view(want[n].shape)
    b = art.bind_into(targets)
    torch.cuda.synchronize()
    for n in names:
        assert torch.equal(targets[n].cpu(), want[n].contiguous()), n
    for g in guards:
        h = g.cpu()
        assert (h[:256] == 0xA5).all() and (h[-256:] == 0xA5).all()
    assert b.data_multihash and b.tensor_dict() is not None


@pytest.mark.gpu
def test_bind_into_with_mapping(cuda_device, artifact):
    from safetensors.torch import load_file
    ref = load_file(artifact)
    p = "model.layers.1.self_attn."
    qkv = torch.empty((256, 128), dtype=torch.bfloat16, device="cuda")
    o_hi = torch.empty((128, 64), dtype=torch.bfloat16, device="cuda")
    gate_up = torch.empty((512, 128), dtype=torch.bfloat16, device="cuda")
    targets = {"qkv": qkv, "o_hi": o_hi, "gate_up": gate_up}
    q = "model.layers.0.mlp."
    plan = [(p + "q_proj.weight", None, "qkv", {"dim": 0, "start": 0, "end": 128}),
            (p + "k_proj.weight", None, "qkv", {"dim": 0, "start": 128, "end": 192}),
            (p + "v_proj.weight", None, "qkv", {"dim": 0, "start": 192, "end": 256}),
            (p + "o_proj.weight", {"dim": 1, "start": 64, "end": 128}, "o_hi", None),
            (q + "gate_proj.weight", None, "gate_up", {"dim": 0, "start": 0, "end": 256}),
            (q + "up_proj.weight", None, "gate_up", {"dim": 0, "start": 256, "end": 512})]
    api.from_disk(artifact).bind_into(targets, mapping=plan)
    torch.cuda.synchronize()
    assert torch.equal(qkv.cpu(), torch.cat([ref[p + "q_proj.weight"], ref[p + "k_proj.weight"],
                                             ref[p + "v_proj.weight"]]))
    assert torch.equal(o_hi.cpu(), ref[p + "o_proj.weight"][:, 64:])
    assert torch.equal(gate_up.cpu(), torch.cat([ref[q + "gate_proj.weight"], ref[q + "up_proj.weight"]]))
    with pytest.raises(api.ArtifactError, match="storage_offset=0"):
        api.from_disk(artifact).bind_into({"o_hi": torch.empty((2, 128, 64), dtype=torch.bfloat16, device="cuda")[1]},
                                          mapping=[(p + "o_proj.weight", {"dim": 1, "start": 64, "end": 128},
                                                    "o_hi", None)])


@pytest.mark.gpu
def test_bind_into_rejects_bad_targets(cuda_device, artifact):
    art = api.from_disk(artifact).subset(["model.norm.weight"])
    with pytest.raises(api.ArtifactError, match="must cover the artifact selection"):
        art.bind_into({"x": torch.empty(128, dtype=torch.bfloat16, device="cuda")})
    with pytest.raises(api.ArtifactError, match="must be CUDA"):
        art.bind_into({"model.norm.weight": torch.empty(128, dtype=torch.bfloat16)})
    with pytest.raises(api.ArtifactError, match="must be torch.bfloat16"):
        art.bind_into({"model.norm.weight": torch.empty(64, dtype=torch.bfloat16, device="cuda")})
    with pytest.raises(api.ArtifactError, match="packing must be"):
        art.bind_into({"model.norm.weight": torch.empty(128, dtype=torch.bfloat16, device="cuda")}, packing="x")


def test_mapped_copy_jobs_three_d_and_scalars(tmp_path):
    """Dim-1 slices of a 3-D tensor (rows of slice x inner elements), a scalar and a 1-D
    split, applied in numpy: every target equals torch slicing of the source."""
    import json as _json
    import struct
    tensors = {"w3": torch.arange(4 * 6 * 5, dtype=torch.int32).view(4, 6, 5),
               "s": torch.tensor(7, dtype=torch.int32), "v": torch.arange(10, dtype=torch.int32)}
    hdr, payload, off = {}, b"", 0
    for n in sorted(tensors):
        b = tensors[n].numpy().tobytes()
        hdr[n] = {"dtype": "I32", "shape": list(tensors[n].shape), "data_offsets": [off, off + len(b)]}
        payload += b
        off += len(b)
    raw = _json.dumps(hdr).encode()
    raw += b" " * ((8 - (8 + len(raw)) % 8) % 8)
    path = tmp_path / "t.safetensors"
    path.write_bytes(struct.pack("<Q", len(raw)) + raw + payload)
    index = build_canonical_index(build_source_index([str(path)]))
    canon = np.zeros(index.total_bytes, np.uint8)
    for n, e in index.entries.items():
        canon[e.offset:e.offset + e.size] = np.frombuffer(tensors[n].numpy().tobytes(), np.uint8)
    mem = torch.zeros(1 << 14, dtype=torch.uint8)
    a = mem[0:4 * 2 * 5 * 4].view(torch.int32).view(4, 2, 5)
    b = mem[1024:1024 + 4 * 4 * 5 * 4].view(torch.int32).view(4, 4, 5)
    sc = mem[4096:4100].view(torch.int32).view(())
    v = mem[8192:8192 + 40].view(torch.int32)
    targets = {"a": a, "b": b, "sc": sc, "v": v}
    plan = [CopyPlanEntry("w3", Range(1, 0, 2), "a", None), CopyPlanEntry("w3", Range(1, 2, 6), "b", None),
            CopyPlanEntry("s", None, "sc", None), CopyPlanEntry("v", Range(0, 5, 10), "v", Range(0, 0, 5)),
            CopyPlanEntry("v", Range(0, 0, 5), "v", Range(0, 5, 10))]
    validate_copy_plan(plan=plan, canonical_index=index,
                       target_tensors={k: torch.empty_like(t) for k, t in targets.items()})
    _apply(mapped_copy_jobs(plan, index, targets, mem.data_ptr()), canon, mem.numpy())
    assert torch.equal(a, tensors["w3"][:, :2]) and torch.equal(b, tensors["w3"][:, 2:])
    assert int(sc) == 7 and torch.equal(v, torch.cat([tensors["v"][5:], tensors["v"][:5]]))
