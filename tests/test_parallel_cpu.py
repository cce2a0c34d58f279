"""Host logic of the multi-GPU layouts on CPU: shard bounds, and the L-sharded top-k
exchange run as two gloo ranks (world size 2) with the oracle standing in for the device
compute.  The merged result must equal the single-process top-k of the whole row."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsa_b200.parallel import LShardedTopK, batch_shard, shard_bounds


def test_shard_bounds_cover_the_range_in_order():
    for length in (1, 7, 131072, 131075):
        for world in (1, 2, 3, 8):
            if length < world:
                continue
            spans = [shard_bounds(length, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == length
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    assert batch_shard(64, 3, 8) == slice(24, 32)
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _oracle_local(queries, weights, keys_shard, k, offset):
    import oracle

    s = np.stack([oracle.full_scores(q, w, kk) for q, w, kk in
                  zip(queries.numpy(), weights.numpy(), keys_shard.numpy())])
    idx, val = oracle.topk_rows(s, k, sorted=False)
    return torch.from_numpy(val), torch.from_numpy(idx.astype(np.int32) + offset)


def _oracle_merge(values, indices, k, sorted_):
    import oracle

    idx, val = oracle.merge_topk(values.numpy(), indices.numpy(), k, sorted=sorted_)
    return torch.from_numpy(idx), torch.from_numpy(val)


def _rank_main(rank, world, port, out_dir, scores_mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        gen = torch.Generator().manual_seed(7)
        b, length, k = 3, 4099, 300
        q = torch.randn(b, 64, 128, generator=gen) / 11
        w = torch.randn(b, 64, generator=gen) / 8
        keys = torch.randn(b, length, 128, generator=gen)
        if scores_mode == "ties":  # whole runs of equal keys -> equal scores across shards
            keys = keys.round()
            keys[:, 1000:3000] = keys[:, 1000:1001]
        start, stop = shard_bounds(length, rank, world)
        sharded = LShardedTopK(k, sorted=True, local_fn=_oracle_local, merge_fn=_oracle_merge)
        idx, val = sharded(q, w, keys[:, start:stop], start)
        if rank == 0:
            np.savez(os.path.join(out_dir, "merged.npz"), idx=idx.numpy(), val=val.numpy(),
                     q=q.numpy(), w=w.numpy(), keys=keys.numpy())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("scores_mode", ["random", "ties"])
def test_l_sharded_topk_two_gloo_ranks_equals_whole_row(tmp_path, scores_mode):
    import oracle

    mp.spawn(_rank_main, args=(2, _free_port(), str(tmp_path), scores_mode), nprocs=2,
             join=True)
    r = np.load(tmp_path / "merged.npz")
    s = np.stack([oracle.full_scores(q, w, kk) for q, w, kk in zip(r["q"], r["w"], r["keys"])])
    want_i, want_v = oracle.topk_rows(s, 300, sorted=True)
    np.testing.assert_array_equal(r["idx"], want_i)
    np.testing.assert_array_equal(r["val"], want_v)
