"""Seeded synthetic safetensors artifacts with Llama-3 shapes (no checkpoints exist offline).

Scheme (fixed, so every run and every machine writes the same bytes):
* tensor k (0-based, in sorted-name order) of an artifact with seed s draws from a
  torch.Generator seeded with ``(s << 32) | k``: ``randn(shape, float32) * 0.02 -> bfloat16``;
  RMSNorm weights (``*norm.weight``) are ones;
* the file is a standard safetensors file (8-byte little-endian header length, JSON header
  padded with spaces to a multiple of 8, then the payload) with tensors stored in sorted-name
  order, which for an all-bf16 model is also the canonical order, so payload == canonical
  bytes (the loader checks this rather than assuming it);
* ``transposed`` names are stored with their two dimensions swapped ([in, out]), as the
  70B benchmark stores one o_proj.
Generation runs on CUDA when available (fast) and on the CPU otherwise; the two devices
produce different (each deterministic) bytes, so fixtures record the device used.
"""
from __future__ import annotations

import json
import os
import struct

import torch

LLAMA3_8B = dict(vocab=128256, hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128, ffn=14336)
LLAMA3_70B = dict(vocab=128256, hidden=8192, layers=80, heads=64, kv_heads=8, head_dim=128, ffn=28672)


def llama_shapes(cfg: dict, transposed=()) -> dict[str, tuple]:
    h, kv = cfg["hidden"], cfg["kv_heads"] * cfg["head_dim"]
    q = cfg["heads"] * cfg["head_dim"]
    shapes = {"model.embed_tokens.weight": (cfg["vocab"], h), "model.norm.weight": (h,),
              "lm_head.weight": (cfg["vocab"], h)}
    for i in range(cfg["layers"]):
        p = f"model.layers.{i}."
        shapes[p + "input_layernorm.weight"] = (h,)
        shapes[p + "post_attention_layernorm.weight"] = (h,)
        shapes[p + "self_attn.q_proj.weight"] = (q, h)
        shapes[p + "self_attn.k_proj.weight"] = (kv, h)
        shapes[p + "self_attn.v_proj.weight"] = (kv, h)
        shapes[p + "self_attn.o_proj.weight"] = (h, q)
        shapes[p + "mlp.gate_proj.weight"] = (cfg["ffn"], h)
        shapes[p + "mlp.up_proj.weight"] = (cfg["ffn"], h)
        shapes[p + "mlp.down_proj.weight"] = (h, cfg["ffn"])
    for name in transposed:
        a, b = shapes[name]
        shapes[name] = (b, a)
    return shapes


def tiny_llama(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=256) -> dict:
    return dict(vocab=vocab, hidden=hidden, layers=layers, heads=heads, kv_heads=kv_heads, head_dim=head_dim, ffn=ffn)


def artifact_bytes(shapes: dict) -> int:
    return sum(2 * _numel(s) for s in shapes.values())


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def tensor_data(name: str, shape, k: int, seed: int, device) -> torch.Tensor:
    if name.endswith("norm.weight"):
        return torch.ones(shape, dtype=torch.bfloat16, device=device)
    g = torch.Generator(device=device)
    g.manual_seed((seed << 32) | k)
    return (torch.randn(shape, generator=g, dtype=torch.float32, device=device) * 0.02).to(torch.bfloat16)


def write_safetensors(path: str, shapes: dict, seed: int, device=None, chunk_bytes: int = 1 << 30) -> dict:
    """Writes the artifact; returns {"path", "payload_offset", "total_bytes", "device"}."""
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    names = sorted(shapes, key=lambda s: s.encode("utf-8"))
    header, off = {}, 0
    for n in names:
        nb = 2 * _numel(shapes[n])
        header[n] = {"dtype": "BF16", "shape": list(shapes[n]), "data_offsets": [off, off + nb]}
        off += nb
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - (8 + len(raw)) % 8) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        pending, pending_bytes = [], 0
        for k, n in enumerate(names):
            t = tensor_data(n, shapes[n], k, seed, device)
            pending.append(t.reshape(-1).view(torch.uint8))
            pending_bytes += t.numel() * 2
            if pending_bytes >= chunk_bytes or k == len(names) - 1:
                buf = torch.cat(pending).cpu().numpy() if len(pending) > 1 else pending[0].cpu().numpy()
                f.write(memoryview(buf))
                pending, pending_bytes = [], 0
    os.replace(tmp, path)
    return {"path": path, "payload_offset": 8 + len(raw), "total_bytes": off, "device": str(device)}


def safetensors_layout(shapes: dict) -> tuple[bytes, dict]:
    """(header bytes incl. the 8-byte length, name -> (payload offset, nbytes)), sorted-name order."""
    names = sorted(shapes, key=lambda s: s.encode("utf-8"))
    header, off, where = {}, 0, {}
    for n in names:
        nb = 2 * _numel(shapes[n])
        header[n] = {"dtype": "BF16", "shape": list(shapes[n]), "data_offsets": [off, off + nb]}
        where[n] = (off, nb)
        off += nb
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - (8 + len(raw)) % 8) % 8)
    return struct.pack("<Q", len(raw)) + raw, where


def write_safetensors_parallel(path: str, shapes: dict, seed: int, world: int, rank: int, device=None,
                               timeout_s: float = 1800.0) -> dict:
    """The same bytes as write_safetensors, written by `world` cooperating processes: rank 0
    writes the header and sizes the file, then every rank generates the tensors k with
    k % world == rank (k in sorted-name order) and writes them in place. Progress is
    coordinated with marker files next to `path`; returns once every rank has finished."""
    import time
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    head, where = safetensors_layout(shapes)
    total = sum(nb for _, nb in where.values())
    tmp = path + ".partial"
    ready = tmp + ".ready"
    if rank == 0:
        for stale in [ready] + [f"{tmp}.done{r}" for r in range(world)]:
            if os.path.exists(stale):
                os.unlink(stale)
        with open(tmp, "wb") as f:
            f.write(head)
            f.truncate(len(head) + total)
        open(ready, "w").close()
    t0 = time.time()
    while not os.path.exists(ready):
        if time.time() - t0 > timeout_s:
            raise TimeoutError("rank 0 did not create the artifact file")
        time.sleep(0.2)
    names = sorted(shapes, key=lambda s: s.encode("utf-8"))
    fd = os.open(tmp, os.O_WRONLY)
    try:
        for k, n in enumerate(names):
            if k % world != rank:
                continue
            t = tensor_data(n, shapes[n], k, seed, device)
            buf = t.reshape(-1).view(torch.uint8).cpu().numpy()
            off = len(head) + where[n][0]
            mv = memoryview(buf)
            done = 0
            while done < len(mv):
                done += os.pwrite(fd, mv[done:], off + done)
    finally:
        os.close(fd)
    open(f"{tmp}.done{rank}", "w").close()
    if rank == 0:
        while not all(os.path.exists(f"{tmp}.done{r}") for r in range(world)):
            if time.time() - t0 > timeout_s:
                raise TimeoutError("a rank did not finish writing the artifact")
            time.sleep(0.2)
        os.replace(tmp, path)
        for m in [ready] + [f"{tmp}.done{r}" for r in range(world)]:
            os.unlink(m)
    return {"path": path, "payload_offset": len(head), "total_bytes": total, "device": str(device)}
