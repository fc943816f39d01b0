"""The batch-sharded project order with the output all-gather fused into the sampler (shard.PeerGather,
td_project_forward_peer): each rank's rows stored into every rank's gathered output over NVLink peer mappings, a
completion signal from each rank's last CTA and a bounded wait per rank. On two GPUs (skipped with fewer): the
gathered output against the unsharded operator on the whole batch, bit for bit, over several calls (the epoch
protocol), ragged and empty shards, float16 / bfloat16 / float32, and replays of a captured CUDA graph. On one GPU:
the wait running out on a peer that never signals ends in an error status and leaves the context usable (the
failure is made on the host side of the protocol: nothing faults or hangs)."""

import datetime
import os
import socket

import pytest
import torch

from cases import make
from marearts_tinydeform_b200 import _native, ma_deform_attn

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errors):
    import torch.distributed as dist
    from marearts_tinydeform_b200 import ma_deform_attn
    from marearts_tinydeform_b200.shard import PeerGather, shard_inputs
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group('gloo', init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        cases = [(3, 33, 8, 32, 256, [(12, 13), (6, 7)], 4, torch.float16),   # ragged: 2 + 1 images
                 (1, 20, 8, 32, 256, [(10, 12), (5, 6)], 4, torch.bfloat16),  # rank 1 has no image
                 (4, 17, 4, 16, 64, [(9, 11), (5, 6)], 4, torch.float32)]
        for B, Q, H, D, C, levels, P, dtype in cases:
            pg = PeerGather(B, Q, H, D, dtype)
            try:
                sets = [[t.cuda() for t in make(B, Q, H, D, C, levels, P, dtype=dtype, seed=40 + s)]
                        for s in range(3)]
                with torch.inference_mode():
                    wants = [ma_deform_attn(*full, mode='project') for full in sets]
                    for call in range(5):
                        got = pg(*shard_inputs(sets[call % 3], rank, world))
                        torch.cuda.synchronize()
                        if not torch.equal(got, wants[call % 3]):
                            err = (got.float() - wants[call % 3].float()).abs().max().item()
                            raise AssertionError(f'rank {rank} {dtype} B={B} call {call}: max |diff| {err}')
                    # two calls per graph (the two buffers), replayed
                    side = torch.cuda.Stream()
                    side.wait_stream(torch.cuda.current_stream())
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.stream(side):
                        with torch.cuda.graph(graph, stream=side):
                            g0 = pg(*shard_inputs(sets[0], rank, world))
                            g1 = pg(*shard_inputs(sets[1], rank, world))
                    torch.cuda.current_stream().wait_stream(side)
                    for _ in range(3):
                        graph.replay()
                        torch.cuda.synchronize()
                        if not (torch.equal(g0, wants[0]) and torch.equal(g1, wants[1])):
                            raise AssertionError(f'rank {rank} {dtype} B={B}: graph replay differs')
                    del graph
                if _native.device_error(clear=True) != 0:
                    raise AssertionError(f'rank {rank}: device error word set')
            finally:
                pg.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent, which fails the test
        errors.put(f'rank {rank}: {exc!r}')
        raise


@pytest.mark.timeout(600)
def test_peer_gather_on_two_gpus(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    import torch.multiprocessing as mp
    ctx = mp.get_context('spawn')
    errors = ctx.Queue()
    port = _free_port()  # both ranks rendezvous on it
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errors)) for r in range(2)]
    env_before = os.environ.get('NCCL_NVLS_ENABLE')
    os.environ['NCCL_NVLS_ENABLE'] = '0'
    try:
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=540)
    finally:
        if env_before is None:
            os.environ.pop('NCCL_NVLS_ENABLE', None)
        else:
            os.environ['NCCL_NVLS_ENABLE'] = env_before
        for p in procs:
            if p.is_alive():
                p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_peer_gather_on_one_rank_without_a_process_group(cuda):
    """No process group: one rank holding the whole batch, the peer sampler storing into the one output. Bit for bit
    the operator's project order over several calls and both buffers: 800 rows (a row a warp), 2,400 (two rows a
    warp, six corner rows in flight a lane: one image a rank in the eight-GPU split of c3) and 19,200 (two rows a warp
    over several waves)."""
    from marearts_tinydeform_b200.shard import PeerGather
    for B, Q, dtype in ((2, 50, torch.float16), (1, 300, torch.bfloat16), (8, 300, torch.bfloat16),
                        (8, 300, torch.float16)):
        H, D, C, levels, P = 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4
        pg = PeerGather(B, Q, H, D, dtype)
        try:
            assert (pg.world, pg.rank) == (1, 0)
            sets = [[t.cuda() for t in make(B, Q, H, D, C, levels, P, dtype=dtype, seed=60 + s)] for s in range(2)]
            with torch.inference_mode():
                for call in range(4):
                    want = ma_deform_attn(*sets[call % 2], mode='project')
                    got = pg(*sets[call % 2])
                    torch.cuda.synchronize()
                    assert torch.equal(got, want), f'B={B} {dtype} call {call}'
            assert _native.device_error(clear=True) == 0
        finally:
            pg.close()


def test_peer_wait_runs_out_on_a_silent_peer(cuda):
    """world = 2 on one control block whose peer slot nothing ever writes: the wait gives up after ~1 ms of clock
    cycles, records the peer-wait code, still advances the epoch, and the context stays usable."""
    from marearts_tinydeform_b200.shard import _DeviceBuffer
    _native.device_error(clear=True)
    ptr, _ = _native.peer_buffer_alloc(_native.PEER_CTRL_BYTES)
    dev = torch.device('cuda', 0)
    try:
        ctrl = torch.as_tensor(_DeviceBuffer(ptr, (16,), '<i4', dev), device=dev)
        _native.test_peer_wait(ptr, 2, 0, 2_000_000, dev)
        torch.cuda.synchronize()
        assert _native.device_error(clear=True) == _native.DEVERR_PEER_WAIT
        assert int(ctrl[8]) == 1  # the epoch still advanced, so the ranks stay in step
        # peer 1 signals the next epoch (written here by the host side of the test): the wait returns at once
        ctrl[1] = 2
        _native.test_peer_wait(ptr, 2, 0, 2_000_000, dev)
        torch.cuda.synchronize()
        assert _native.device_error(clear=True) == 0
        assert int(ctrl[8]) == 2
        x = torch.ones(1000, device='cuda')
        assert float(x.sum()) == 1000.0
    finally:
        _native.peer_buffer_close(ptr, False)
