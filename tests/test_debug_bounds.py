"""The checked build (_tinydeform_debug.so, -DTD_DEBUG_BOUNDS): every corner token is re-tested against [0, N) where
a kernel reads or writes its row, and a token outside it is recorded in the device error word (code 4) and skipped.
On tiny shapes of every kind -- random, far outside, on pixel borders, with a padding mask, both kernel policies,
every dtype -- both orders and the backward must run with no such record and match the oracle."""

import ctypes
import os

import pytest
import torch

from cases import boundary_case, make, to, upcast
from marearts_tinydeform_b200 import _native, build, ma_deform_attn
from oracle import deform_oracle as O

TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (3e-3, 3e-3), torch.bfloat16: (2e-2, 2e-2),
       torch.float64: (1e-12, 1e-10)}


def test_checked_library_exports_the_same_symbols():
    build.build(debug=True)
    lib = ctypes.CDLL(build.DEBUG_LIB)
    for name in _native.SIGNATURES:
        assert hasattr(lib, name), name


@pytest.fixture
def checked(cuda):
    """_native's entry points bound to the checked library for the test's duration."""
    lib = ctypes.CDLL(build.DEBUG_LIB)
    for name, (res, args) in _native.SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    saved = _native._lib
    _native._lib = lib
    code = ctypes.c_uint(0)
    lib.td_device_error(1, ctypes.byref(code), None, 0)
    yield lib
    _native._lib = saved


def _error_word(lib):
    torch.cuda.synchronize()
    code = ctypes.c_uint(0)
    assert lib.td_device_error(1, ctypes.byref(code), None, 0) == 0
    return code.value


@pytest.mark.gpu
@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16, torch.float64])
def test_no_token_leaves_its_map(checked, dtype):
    cases = [make(2, 9, 4, 32, 256, [(7, 9), (4, 5)], 4, dtype=dtype, seed=3),        # tensor-core widths
             make(1, 6, 2, 8, 16, [(6, 7), (3, 4)], 2, dtype=dtype, seed=4, spread=200.0),  # far outside
             make(2, 5, 3, 10, 30, [(5, 7), (3, 4)], 4, dtype=dtype, seed=5),          # odd widths
             make(1, 40, 8, 32, 256, [(20, 20), (10, 10)], 4, dtype=dtype, seed=6),    # rows of 512+ bytes
             boundary_case(dtype)]
    for policy in (_native.POLICY_BEST, _native.POLICY_CUDA_CORES):
        prev = checked.td_set_kernel_policy(policy)
        try:
            for args in cases:
                N = args[0].shape[1]
                mask = torch.rand(args[0].shape[0], N, generator=torch.Generator().manual_seed(N)) < 0.2
                for m in (None, mask):
                    ref = torch.from_numpy(O.ma_deform_attn_oracle(*[t if t is None else t.cpu() for t in upcast(args)],
                                                                   value_padding_mask=m))
                    with torch.inference_mode():
                        for mode in ('fused', 'project'):
                            got = ma_deform_attn(*to(args, 'cuda'), mode=mode,
                                                 value_padding_mask=None if m is None else m.cuda()).double().cpu()
                            assert torch.allclose(got, ref, atol=TOL[dtype][0], rtol=TOL[dtype][1]), (mode, policy)
                    assert _error_word(checked) == 0
        finally:
            checked.td_set_kernel_policy(prev)


@pytest.mark.gpu
def test_no_token_leaves_its_map_in_the_backward(checked):
    for dtype in (torch.float32, torch.float16, torch.float64):
        args = make(1, 7, 2, 16, 32, [(6, 7), (3, 4)], 4, dtype=dtype, seed=8, spread=2.0)
        x = [t.cuda().requires_grad_(True) if t is not None and t.is_floating_point() else
             (t.cuda() if t is not None else None) for t in args]
        for mode in ('project', 'fused'):
            out = ma_deform_attn(*x, mode=mode)
            out.square().sum().backward()
            assert _error_word(checked) == 0
            for t in x:
                if t is not None and t.grad is not None:
                    assert torch.isfinite(t.grad).all()
                    t.grad = None
