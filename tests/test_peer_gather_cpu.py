"""Host logic of shard.PeerGather on world-size-2 gloo groups on CPU, with the library's device calls replaced by
recording fakes: the IPC handles travel to every rank, each rank's table holds its own buffers at its own rank and
the peers' mappings elsewhere, calls pass batch_range's first image and alternate the output buffers, a shard of the
wrong size is refused before any device call, and close() unmaps the peers' buffers, waits for every rank, then
frees its own."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    from marearts_tinydeform_b200 import _native, shard
    log = []
    counter = [0]

    def alloc(nbytes):
        counter[0] += 1
        ptr = 1000 * (rank + 1) + counter[0]
        log.append(('alloc', ptr, nbytes))
        return ptr, f'r{rank}b{counter[0]}'.encode().ljust(64, b'\0')

    def open_(handle):
        name = bytes(handle).rstrip(b'\0').decode()
        ptr = 50000 + 1000 * int(name[1]) + int(name[3:])
        log.append(('open', name, ptr))
        return ptr

    def close(ptr, opened):
        log.append(('close', ptr, opened))

    def forward(*args, **kw):
        log.append(('forward', args[7], args[8], list(args[9]), list(args[10])))

    _native.peer_buffer_alloc, _native.peer_buffer_open = alloc, open_
    _native.peer_buffer_close, _native.project_forward_peer = close, forward
    shard._device_view = lambda ptr, shape, dtype, device: torch.full(shape, ptr, dtype=torch.float64)
    dist.init_process_group('gloo', init_method=f'tcp://127.0.0.1:{port}', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        pg = shard.PeerGather(3, 5, 2, 16, torch.float32, device='cpu', buffers=2)
        mine = 2 if rank == 0 else 1  # batch_range(3, 2, rank)
        mem = torch.zeros(mine, 7, 32)
        loc = torch.zeros(mine, 5, 2, 1, 2, 2)
        att = torch.zeros(mine, 5, 2, 1, 2)
        outs = [pg(mem, None, None, None, None, loc, att) for _ in range(3)]
        with pytest.raises(ValueError):
            pg(torch.zeros(mine + 1, 7, 32), None, None, None, None, loc, att)
        pg.close()
        q.put((rank, log, [float(o.flatten()[0]) for o in outs]))
    finally:
        dist.destroy_process_group()


def test_peer_gather_host_logic_on_two_gloo_ranks():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        rank, log, firsts = q.get(timeout=120)
        got[rank] = (log, firsts)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        log, firsts = got[rank]
        allocs = [e for e in log if e[0] == 'alloc']
        assert len(allocs) == 3  # two outputs, one control block
        opens = [e for e in log if e[0] == 'open']
        peer = 1 - rank
        assert [e[1] for e in opens] == [f'r{peer}b1', f'r{peer}b2', f'r{peer}b3']
        fwd = [e for e in log if e[0] == 'forward']
        assert len(fwd) == 3
        first_image = 0 if rank == 0 else 2
        own = [a[1] for a in allocs]
        peer_ptrs = [e[2] for e in opens]
        for call, (_, fi, rk, outs, ctrls) in enumerate(fwd):
            k = call % 2
            assert fi == first_image and rk == rank
            assert outs[rank] == own[k] and outs[peer] == peer_ptrs[k]
            assert ctrls[rank] == own[2] and ctrls[peer] == peer_ptrs[2]
        # the returned tensors are the two own buffers in turn
        assert firsts == [own[0], own[1], own[0]]
        # peers' mappings closed before this rank's own buffers are freed
        closes = [e for e in log if e[0] == 'close']
        assert [c[2] for c in closes] == [True, True, True, False, False, False]
        assert sorted(c[1] for c in closes[3:]) == sorted(own)
