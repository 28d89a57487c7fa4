"""The SDK mirror (tensorcast_b200.api): from_disk / subset / view / tensor_dict, checked
against the safetensors library's own reader (CPU parts need no GPU)."""
import json
import os

import numpy as np
import pytest
import torch

from tensorcast_b200 import api
from tensorcast_b200.synthetic import llama_shapes, tiny_llama, write_safetensors


@pytest.fixture(scope="module")
def artifact(tmp_path_factory):
    d = tmp_path_factory.mktemp("art")
    path = os.path.join(d, "model.safetensors")
    write_safetensors(path, llama_shapes(tiny_llama(layers=2, hidden=64, ffn=128, vocab=512)), 4, device="cpu")
    return path


def test_from_disk_index_matches_safetensors_header(artifact):
    from safetensors import safe_open
    art = api.from_disk(artifact)
    with safe_open(artifact, framework="pt") as f:
        names = sorted(f.keys())
        assert list(art.index.entries) == names
        for n in names:
            assert tuple(f.get_slice(n).get_shape()) == art.index.entries[n].shape
    offs = [e.offset for e in art.index.entries.values()]
    assert offs == sorted(offs) and all(o % 8 == 0 for o in offs)
    # canonical index JSON in the reference's [offset,size,shape,stride,dtype,storage_offset] form
    j = json.loads(art.canonical_index_json)
    first = names[0]
    assert j[first][0] == 0 and j[first][4] == "torch.bfloat16" and j[first][5] == 0


def test_view_validation_mirrors_reference(artifact):
    art = api.from_disk(artifact)
    with pytest.raises(ValueError, match="Slice step must be 1"):
        art.view(slices={"lm_head.weight": slice(0, 10, 2)})
    with pytest.raises(ValueError, match="unknown tensor"):
        art.subset(["nope"])
    with pytest.raises(ValueError, match="out of range"):
        art.view(slices={"model.norm.weight": (1, slice(0, 2))})
    with pytest.raises(api.ArtifactError, match="does not exist"):
        api.from_disk(artifact + ".missing")


@pytest.mark.gpu
def test_tensor_dict_matches_safetensors(cuda_device, artifact):
    from safetensors.torch import load_file
    ref = load_file(artifact)
    names = ["lm_head.weight", "model.layers.0.mlp.down_proj.weight", "model.norm.weight",
             "model.layers.1.self_attn.o_proj.weight"]
    art = api.from_disk(artifact).subset(names).view(
        slices={"lm_head.weight": slice(128, 256), "model.layers.0.mlp.down_proj.weight": (1, slice(32, 96))},
        transpose={"model.layers.1.self_attn.o_proj.weight": [(0, 1)]})
    got = art.tensor_dict(device="cuda:0")
    assert list(got) == names
    assert torch.equal(got["lm_head.weight"].cpu(), ref["lm_head.weight"][128:256])
    assert torch.equal(got["model.layers.0.mlp.down_proj.weight"].cpu(),
                       ref["model.layers.0.mlp.down_proj.weight"][:, 32:96])
    assert torch.equal(got["model.norm.weight"].cpu(), ref["model.norm.weight"])
    assert torch.equal(got["model.layers.1.self_attn.o_proj.weight"].cpu(),
                       ref["model.layers.1.self_attn.o_proj.weight"].t().contiguous())
    full = api.from_disk(artifact).tensor_dict(device="cuda:0")
    for n, t in ref.items():
        assert torch.equal(full[n].cpu(), t)


@pytest.mark.gpu
def test_descriptor_verification(cuda_device, artifact, tmp_path):
    from oracle import oracle
    art = api.from_disk(artifact)
    art.tensor_dict(device="cuda:0")
    good = art.data_multihash
    # the GPU entry's data multihash of the canonical bytes (adaptive leaf policy)
    start = min(s.file_offset for s in art.index.sources.values())
    canon = np.fromfile(artifact, dtype=np.uint8)[start:start + art.index.total_bytes]
    assert good == oracle.multihash_gpu_semantics(canon)
    desc = os.path.join(os.path.dirname(artifact), "artifact_descriptor.json")
    try:
        with open(desc, "w") as f:
            json.dump({"data_multihash": good}, f)
        api.from_disk(artifact).tensor_dict(device="cuda:0")
        bad = oracle.multihash(bytes(32))
        with open(desc, "w") as f:
            json.dump({"data_multihash": bad}, f)
        with pytest.raises(api.ArtifactError, match="ARTIFACT_ID_MISMATCH") as ei:
            api.from_disk(artifact).tensor_dict(device="cuda:0")
        assert ei.value.status_code == "DATA_LOSS"
    finally:
        os.unlink(desc)


def test_canonical_index_multi_file_and_float8(tmp_path):
    """test_safetensors_loading.py:12-67: canonical offsets are coalesced by sorted tensor
    name across files (not file order), and float8 dtypes map to the torch names."""
    from safetensors.torch import save_file
    from tensorcast_b200.artifact import build_canonical_index, build_source_index, safetensors_files
    d = tmp_path / "st"
    d.mkdir()
    save_file({"t": torch.arange(256, dtype=torch.uint8)}, str(d / "weights.safetensors"))
    idx = build_canonical_index(build_source_index(safetensors_files(str(d))))
    e = idx.entries["t"]
    assert (e.offset, e.size, list(e.shape), list(e.stride), e.dtype, e.storage_offset) == \
        (0, 256, [256], [1], "torch.uint8", 0)
    save_file({"u": torch.arange(16, dtype=torch.uint8)}, str(d / "extra.safetensors"))
    idx = build_canonical_index(build_source_index(safetensors_files(str(d))))
    assert [(n, e.offset, e.size) for n, e in idx.entries.items()] == [("t", 0, 256), ("u", 256, 16)]
    f8 = tmp_path / "f8"
    f8.mkdir()
    save_file({"fp8_e4m3": torch.zeros(8, dtype=torch.float8_e4m3fn),
               "fp8_e5m2": torch.ones(8, dtype=torch.float8_e5m2)}, str(f8 / "weights.safetensors"))
    idx = build_canonical_index(build_source_index(safetensors_files(str(f8))))
    assert idx.entries["fp8_e4m3"].dtype == "torch.float8_e4m3fn"
    assert idx.entries["fp8_e5m2"].dtype == "torch.float8_e5m2"
    assert (idx.entries["fp8_e4m3"].offset, idx.entries["fp8_e4m3"].size) == (0, 8)
    assert (idx.entries["fp8_e5m2"].offset, idx.entries["fp8_e5m2"].size) == (8, 8)


def test_reader_threads_shared_by_the_hosts_ranks(monkeypatch):
    """File staging spreads the host's CPUs over the ranks that stage at once: all of them for
    one rank, CPUs / LOCAL_WORLD_SIZE for one process per GPU, CPUs / world for rank threads of
    one process; never fewer than 2 or more than 32 per rank."""
    monkeypatch.setattr(api.os, "sched_getaffinity", lambda pid: set(range(48)), raising=False)
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    assert api._reader_threads(1, 0) == 32
    monkeypatch.setattr(api, "_process_model", lambda world, rank: True)
    assert api._reader_threads(8, 3) == 6
    monkeypatch.setattr(api, "_process_model", lambda world, rank: False)
    assert api._reader_threads(4, 1) == 12
    assert api._reader_threads(64, 0) == 2
