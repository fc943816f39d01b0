"""The allocation-free project order (td_project_forward_noalloc) against the workspace entry point.

Some callers cannot allocate device memory while running the operator: plugins inside an inference host that owns
all device memory, real-time loops that cannot afford cudaMalloc's synchronisation, plain C hosts without a caching
allocator. For them the library keeps the projected value in a fixed device array of TD_NOALLOC_SCRATCH_BYTES.
This file is collected last on purpose, and its tests also pass alone in a fresh process.
"""

import ctypes

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
