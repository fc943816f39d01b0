"""The allocation-free project order (td_project_forward_noalloc) against the workspace entry point.

Some callers cannot allocate device memory while running the operator: plugins inside an inference host that owns
all device memory, real-time loops that cannot afford cudaMalloc's synchronisation, plain C hosts without a caching
allocator. For them the library keeps the projected value in a fixed device array of TD_NOALLOC_SCRATCH_BYTES.
This file is collected last on purpose, and its tests also pass alone in a fresh process.
"""

import ctypes
import os
import subprocess
import sys
import textwrap

import pytest
import torch

from marearts_tinydeform_b200 import _native, workloads

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20  # TD_NOALLOC_SCRATCH_BYTES in include/tinydeform.h
TOL = {torch.float16: (3e-3, 3e-3), torch.bfloat16: (2e-2, 2e-2), torch.float32: (2e-5, 1e-4)}


def _args(inputs):
    mem, w, b, shapes, starts, loc, attn = inputs
    B, Q, H, L, P = loc.shape[:5]
    N, C = mem.shape[1:]
    return mem, w, b, shapes, starts, loc, attn, (B, Q, N, C, H, w.shape[0], L, P)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def run_noalloc(lib, inputs, out):
    mem, w, b, shapes, starts, loc, attn, sizes = _args(inputs)
    err = ctypes.create_string_buffer(512)
    rc = lib.td_project_forward_noalloc(_native.DTYPE_CODE[mem.dtype], _p(mem), _p(w), _p(b), _p(shapes), _p(starts),
                                        _p(loc), _p(attn), _p(out), *sizes,
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), err, 512)
    return rc, err.value.decode()


def run_workspace(lib, inputs, out):
    mem, w, b, shapes, starts, loc, attn, sizes = _args(inputs)
    B, Q, N, C, H, HD, L, P = sizes
    code = _native.DTYPE_CODE[mem.dtype]
    ws_bytes = lib.td_project_workspace_bytes(code, B, N, HD)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=mem.device)
    err = ctypes.create_string_buffer(512)
    rc = lib.td_project_forward(code, _p(mem), _p(w), _p(b), _p(shapes), _p(starts), _p(loc), _p(attn), _p(out),
                                *sizes, _p(ws), ws_bytes, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                err, 512)
    torch.cuda.synchronize()
    return rc, err.value.decode()


@pytest.mark.parametrize('name,dtype', [('c1h', torch.float16), ('c2', torch.bfloat16), ('c1', torch.float32)])
def test_no_alloc_matches_the_workspace_entry_point(cuda, name, dtype):
    lib = _native.load()
    atol, rtol = TOL[dtype]
    first = [None if t is None else t.to(cuda) for t in workloads.make_inputs(name, seed=0, dtype=dtype)]
    second = [None if t is None else t.to(cuda) for t in workloads.make_inputs(name, seed=1, dtype=dtype)]
    for inputs in (first, second):  # two calls in a row: the scratch holds the first call's value when the second runs
        B, Q = inputs[5].shape[:2]
        HD = inputs[1].shape[0]
        want = torch.empty(B, Q, HD, dtype=dtype, device=cuda)
        got = torch.full((B, Q, HD), float('nan'), dtype=dtype, device=cuda)
        assert run_workspace(lib, inputs, want) == (0, '')
        assert run_noalloc(lib, inputs, got) == (0, '')
        torch.cuda.synchronize()
        assert torch.allclose(got.float(), want.float(), atol=atol, rtol=rtol), name
    assert _native.device_error(clear=False) == 0


def test_no_alloc_rejects_what_does_not_fit(cuda):
    lib = _native.load()
    inputs = [None if t is None else t.to(cuda) for t in workloads.make_inputs('c1h', seed=0, B=4)]
    out = torch.empty(4, 300, 256, dtype=torch.float16, device=cuda)
    need = lib.td_project_workspace_bytes(_native.TD_F16, 4, 8400, 256)
    assert need > SCRATCH_BYTES
    rc, msg = run_noalloc(lib, inputs, out)
    assert rc == 3 and str(need) in msg and str(SCRATCH_BYTES) in msg


def test_no_alloc_takes_no_device_memory(cuda):
    """After a first call (which looks up the scratch array and loads the kernels), a call changes neither torch's
    allocator nor the device's free memory."""
    lib = _native.load()
    inputs = [None if t is None else t.to(cuda) for t in workloads.make_inputs('c1h', seed=2)]
    out = torch.empty(1, 300, 256, dtype=torch.float16, device=cuda)
    assert run_noalloc(lib, inputs, out) == (0, '')
    torch.cuda.synchronize()
    allocated, free = torch.cuda.memory_allocated(cuda), torch.cuda.mem_get_info(cuda)[0]
    for _ in range(3):
        assert run_noalloc(lib, inputs, out) == (0, '')
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(cuda) == allocated
    assert torch.cuda.mem_get_info(cuda)[0] == free


def test_no_alloc_rejects_bad_arguments_before_the_device(cuda):
    lib = _native.load()
    inputs = [None if t is None else t.to(cuda) for t in workloads.make_inputs('c2', seed=0, Q=8)]
    mem, w, b, shapes, starts, loc, attn, sizes = _args(inputs)
    B, Q, N, C, H, HD, L, P = sizes
    out = torch.empty(B, Q, HD, dtype=mem.dtype, device=cuda)
    err = ctypes.create_string_buffer(512)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptrs = [_p(t) for t in (mem, w, b, shapes, starts, loc, attn, out)]
    assert lib.td_project_forward_noalloc(9, *ptrs, *sizes, stream, err, 512) == 1  # unknown dtype code
    assert lib.td_project_forward_noalloc(_native.TD_F16, *ptrs, B, Q, N, C, 3, HD, L, P, stream, err, 512) == 1
    # B * N * HD * 2 wraps a 64-bit size: rejected as too large, not wrapped below the limit
    rc = lib.td_project_forward_noalloc(_native.TD_F16, *ptrs, 1, 1, 2 ** 31 - 1, C, H, 1 << 40, L, P, stream, err,
                                        512)
    assert rc == 3 and 'SIZE_MAX' in err.value.decode()
    assert _native.device_error(clear=False) == 0


FIRST_CALL_UNDER_CAPTURE = textwrap.dedent("""
    import ctypes, sys, warnings
    import torch
    sys.path[:0] = [{root!r}, {tests!r}]
    from marearts_tinydeform_b200 import _native, workloads
    from test_zz_no_alloc import run_noalloc, run_workspace
    lib = _native.load()
    dev = torch.device('cuda', 0)
    inputs = [None if t is None else t.to(dev) for t in workloads.make_inputs('c1h', seed=3)]
    want = torch.empty(1, 300, 256, dtype=torch.float16, device=dev)
    got = torch.full((1, 300, 256), float('nan'), dtype=torch.float16, device=dev)
    assert run_workspace(lib, inputs, want) == (0, '')
    # the first call of this process on the device comes while the stream captures: refused, nothing recorded
    side, graph = torch.cuda.Stream(), torch.cuda.CUDAGraph()
    with warnings.catch_warnings():
        warnings.simplefilter('ignore')  # torch warns that the captured graph is empty
        with torch.cuda.graph(graph, stream=side):
            rc, msg = run_noalloc(lib, inputs, got)
    assert rc == 2 and 'before any stream capture' in msg, (rc, msg)
    del graph
    # the failed lookup was not remembered: the next call, outside capture, succeeds
    assert run_noalloc(lib, inputs, got) == (0, '')
    torch.cuda.synchronize()
    assert torch.allclose(got.float(), want.float(), atol=3e-3, rtol=3e-3)
    assert _native.device_error(clear=False) == 0
    print('ok')
""")


def test_no_alloc_first_call_under_capture_is_refused_then_retried(cuda):
    """A first call made while its stream captures cannot look up the scratch array: it must fail cleanly and must
    not poison later calls. Run in a fresh process, where that call really is the first on the device."""
    here = os.path.dirname(os.path.abspath(__file__))
    code = FIRST_CALL_UNDER_CAPTURE.format(root=os.path.dirname(here), tests=here)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(torch.cuda.current_device()))
    if 'CUDA_VISIBLE_DEVICES' in os.environ:  # already remapped: keep the parent's view
        env['CUDA_VISIBLE_DEVICES'] = os.environ['CUDA_VISIBLE_DEVICES']
    res = subprocess.run([sys.executable, '-c', code], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0 and res.stdout.strip().endswith('ok'), res.stdout[-2000:] + res.stderr[-2000:]
