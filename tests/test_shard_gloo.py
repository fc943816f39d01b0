"""Batch sharding across ranks, run as world_size-2 gloo process groups on CPU (the multi-GPU host logic):
shard boundaries, per-rank results, the optional output all-gather with ragged and empty shards, and a rank that
fails before the collective (the others get an error from the short process-group timeout instead of hanging)."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cases import make
from marearts_tinydeform_b200 import ma_deform_attn_reference
from marearts_tinydeform_b200.shard import batch_range, ma_deform_attn_sharded, shard_inputs


def test_batch_range_covers_the_batch_once():
    for batch in range(0, 13):
        for world in (1, 2, 3, 4, 8):
            spans = [batch_range(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [s[1] - s[0] for s in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        batch_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, mode, results):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        torch.set_num_threads(1)
        full = make(batch, 7, 2, 8, 16, [(6, 7), (3, 4)], 2, seed=11)
        local = shard_inputs(full, rank, world)
        with torch.inference_mode():
            mine = ma_deform_attn_sharded(*local, gather=False)
            every = ma_deform_attn_sharded(*local, gather=True)
            want = ma_deform_attn_reference(*full)
        start, stop = batch_range(batch, world, rank)
        ok_local = mine.shape[0] == stop - start and torch.allclose(mine, want[start:stop], atol=1e-6)
        ok_all = every.shape == want.shape and torch.allclose(every, want, atol=1e-6)
        # the value padding mask is sliced with the batch
        mask = torch.rand(batch, full[0].shape[1], generator=torch.Generator().manual_seed(5)) < 0.3
        local_m = shard_inputs(full + [mask], rank, world)
        with torch.inference_mode():
            masked = ma_deform_attn_sharded(*local_m[:7], gather=True, value_padding_mask=local_m[7])
            want_m = ma_deform_attn_reference(*full, value_padding_mask=mask)
        ok_all = ok_all and masked.shape == want_m.shape and torch.allclose(masked, want_m, atol=1e-6)
        # the known split (no size exchange): same result, and a shard that does not match the split is refused
        with torch.inference_mode():
            known = ma_deform_attn_sharded(*local, gather=True, global_batch=batch)
        ok_all = ok_all and known.shape == want.shape and torch.allclose(known, want, atol=1e-6)
        try:
            with torch.inference_mode():
                ma_deform_attn_sharded(*local, gather=True, global_batch=batch + world)
            ok_all = False
        except ValueError:
            pass
        results[rank] = (bool(ok_local), bool(ok_all))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('batch', [4, 3, 1])
def test_sharded_results_match_the_whole_batch(batch):
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(world, _free_port(), batch, 'auto', results), nprocs=world, join=True)
        assert dict(results) == {0: (True, True), 1: (True, True)}


def _failing_worker(rank, world, port, results):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    try:
        full = make(2, 5, 2, 8, 16, [(6, 7)], 2, seed=3)
        local = shard_inputs(full, rank, world)
        if rank == 1:
            results[rank] = 'raised'
            raise RuntimeError('rank 1 fails before the collective')
        try:
            with torch.inference_mode():
                ma_deform_attn_sharded(*local, gather=True)
            results[rank] = 'completed'
        except Exception as exc:  # the peer never joins: the gloo timeout ends the collective with an error
            results[rank] = 'error: ' + type(exc).__name__
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_a_failed_rank_ends_the_gather_with_an_error():
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        with pytest.raises(Exception):
            mp.spawn(_failing_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        assert results.get(1) == 'raised'
        assert str(results.get(0, '')).startswith('error')
