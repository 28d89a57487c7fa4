"""Generate the committed golden fixtures for the content-hashing path.

Run from the repository root:  python tests/golden/make_golden.py

The fixtures are produced WITHOUT the C oracle, so that they can pin it: leaf
digests come from Python's ``hashlib.sha256`` (backed by the same OpenSSL
libcrypto that the reference calls in core/common/artifact_hash_cpu.cc:161-196),
and the Merkle reduction and multihash encoding below are a separate, pure-Python
restatement of artifact_hash_cpu.cc:198-254 (tree: pairwise, odd node promoted
unchanged; multihash: 'b' + RFC 4648 base32, lower case, unpadded, of 0x12 0x20 || root).

Inputs are seeded: ``numpy.random.default_rng(seed).integers(0, 256, size, uint8)``.
"""
from __future__ import annotations

import base64
import hashlib
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def seeded_bytes(seed: int, size: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, size=size, dtype=np.uint8)


def sha256_bytes(b: bytes) -> bytes:
    # artifact_hash_cpu.cc:161-164: empty -> 32 zero bytes
    return bytes(32) if len(b) == 0 else hashlib.sha256(b).digest()


def leaf_digests(buf: np.ndarray, leaf: int) -> list[bytes]:
    mv = memoryview(buf)
    return [sha256_bytes(bytes(mv[i:i + leaf])) for i in range(0, buf.size, leaf)]


def tree_root(leaves: list[bytes]) -> bytes:
    level = list(leaves)
    while len(level) > 1:
        nxt = []
        for i in range(0, len(level), 2):
            nxt.append(sha256_bytes(level[i] + level[i + 1]) if i + 1 < len(level) else level[i])
        level = nxt
    return level[0]


def multihash(digest: bytes) -> str:
    return "b" + base64.b32encode(b"\x12\x20" + digest).decode("ascii").lower().rstrip("=")


SMALL_SIZES = [1, 3, 55, 56, 57, 63, 64, 65, 119, 120, 121, 127, 128, 129, 191, 192, 1000, 4096, 4097,
               65536 + 55, 200_003, 1 << 20]
SMALL_LEAVES = [64, 128, 192, 4096, 65536, 524288]


def main() -> None:
    out: dict = {"generator": "numpy.random.default_rng(seed).integers(0,256,size,dtype=uint8)"}

    # Small odd-sized cases: every (size, leaf) pair, seed = size.
    cases = []
    for size in SMALL_SIZES:
        buf = seeded_bytes(size, size)
        for leaf in SMALL_LEAVES:
            d = leaf_digests(buf, leaf)
            root = tree_root(d)
            cases.append({"seed": size, "size": size, "leaf": leaf, "n_leaves": len(d),
                          "first_leaf": d[0].hex(), "last_leaf": d[-1].hex(),
                          "root": root.hex(), "multihash": multihash(root)})
    out["small"] = cases

    # the 1 GiB hash-parity case: seed 0, 4 MiB leaves (256 digests) and the reference GPU
    # policy's 512 KiB leaves (2048 digests).
    c1 = seeded_bytes(0, 1 << 30)
    c1_entries = []
    for leaf, fname in ((4 << 20, "c1_seed0_1gib_leaf4mib.digests.bin"),
                        (512 << 10, "c1_seed0_1gib_leaf512kib.digests.bin")):
        d = leaf_digests(c1, leaf)
        root = tree_root(d)
        with open(os.path.join(HERE, fname), "wb") as f:
            f.write(b"".join(d))
        c1_entries.append({"seed": 0, "size": 1 << 30, "leaf": leaf, "n_leaves": len(d),
                           "digests_file": fname, "root": root.hex(), "multihash": multihash(root)})
    out["c1"] = c1_entries

    with open(os.path.join(HERE, "hash_golden.json"), "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
