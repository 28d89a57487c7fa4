"""Paged KV gather + per-sequence hash (the paged-KV benchmark): workload construction on the
CPU, and on the GPU every gathered sequence and its multihash against the numpy/OpenSSL
oracle (oracle/kv.py)."""
import numpy as np
import pytest
import torch

from tensorcast_b200 import kvcache


def test_workload_matches_config_rules():
    w = kvcache.workload(seed=3)
    assert w.planes == 64 and w.pool_pages == 65536
    pages = -(-w.seq_tokens.astype(np.int64) // 16)
    assert int(pages.sum()) == int(w.page_offsets[-1]) <= 65536
    lens = np.random.default_rng(3).integers(64, 4097, size=4096)
    assert (w.seq_tokens == lens[: w.n_seq]).all()                   # drawn in order
    nxt = -(-int(lens[w.n_seq]) // 16)
    assert int(pages.sum()) + nxt > 65536                             # stopped when the pool is full
    assert np.unique(w.page_table).size == w.page_table.size         # every slot used once
    assert (w.page_table == np.random.default_rng(3).permutation(65536)[: w.page_table.size]).all()
    shards = [w.shard(8, r) for r in range(8)]
    assert sum(s.n_seq for s in shards) == w.n_seq
    assert sorted(np.concatenate([s.page_table for s in shards]).tolist()) == sorted(w.page_table.tolist())


def test_plan_leaf_tables():
    w = kvcache.workload(seed=5, planes=4, pool_pages=256, max_seqs=40, min_tokens=1, max_tokens=200,
                         token_bytes=256)
    p = kvcache.plan(w, leaf=4096)
    sb = w.seq_bytes()
    for i in range(w.n_seq):
        a, b = int(p.seg_first[i]), int(p.seg_first[i + 1])
        assert int(p.leaf_lengths[a:b].sum()) == int(sb[i])
        assert int(p.leaf_offsets[a]) == int(p.out_offsets[i])
        assert (p.leaf_lengths[a:b - 1] == 4096).all()
    assert (p.out_offsets % 256 == 0).all()


@pytest.mark.gpu
@pytest.mark.parametrize("token_bytes,leaf", [(256, 4096), (2048, 2 << 20), (96, 1000)])
def test_gather_and_hash_match_oracle(cuda_device, token_bytes, leaf):
    from oracle import kv as okv
    w = kvcache.workload(seed=11, planes=4, pool_pages=384, max_seqs=64, min_tokens=1, max_tokens=700,
                         token_bytes=token_bytes)
    pool = kvcache.make_pool(w, seed=11)
    g = kvcache.KvGatherHash(w, leaf=leaf)
    g.run(pool)
    torch.cuda.synchronize()
    g.check_status()
    host_pool = pool.cpu().numpy()
    mh = g.multihashes()
    for i in range(w.n_seq):
        slots = w.page_table[w.page_offsets[i]:w.page_offsets[i + 1]]
        want = okv.gather_sequence(host_pool, w.planes, w.pool_pages, w.page_tokens, w.token_bytes, slots,
                                   int(w.seq_tokens[i]))
        assert (g.sequence(i).cpu().numpy() == want).all(), i
        assert mh[i] == okv.sequence_multihash(want, leaf), i


@pytest.mark.gpu
def test_gather_reports_bad_page_table_entries(cuda_device):
    w = kvcache.workload(seed=2, planes=2, pool_pages=64, max_seqs=8, min_tokens=1, max_tokens=100, token_bytes=64)
    w.page_table[0] = 1000  # a slot outside the pool: the kernel skips it and reports code 1
    pool = kvcache.make_pool(w, seed=2)
    g = kvcache.KvGatherHash(w, leaf=4096)
    g.run(pool)
    torch.cuda.synchronize()
    assert int(g.status.item()) == 1
    with pytest.raises(Exception, match="outside the pool"):
        g.check_status()
