"""The C-ABI library: it loads without a GPU, exports exactly what include/tinydeform.h declares, and rejects bad
arguments before touching the device."""

import ctypes
import os
import re

import pytest

from marearts_tinydeform_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'tinydeform.h')


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r'TD_API\s+[\w\s\*]*?\b(td_\w+)\s*\(', text)


@pytest.fixture(scope='module')
def lib():
    from marearts_tinydeform_b200 import build
    build.build()
    return _native.load()


def test_header_declares_the_bound_symbols():
    assert sorted(declared_symbols()) == sorted(_native.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_argument_counts_match_the_header():
    text = open(HEADER).read()
    for name, (_, argtypes) in _native.SIGNATURES.items():
        m = re.search(r'TD_API[^;(]*\b' + name + r'\s*\(([^)]*)\)', text, re.S)
        params = [p for p in m.group(1).split(',') if p.strip() and p.strip() != 'void']
        assert len(params) == len(argtypes), name


def test_version_and_workspace(lib):
    assert lib.td_version().decode().startswith('0.1.1')
    assert lib.td_project_workspace_bytes(_native.TD_F16, 2, 100, 256) == 2 * 100 * 256 * 2 + 256
    assert lib.td_project_workspace_bytes(_native.TD_F32, 1, 10, 8) == 10 * 8 * 4 + 256
    assert lib.td_project_workspace_bytes(99, 1, 10, 8) == 0


def _err():
    return ctypes.create_string_buffer(256)


def call_fused(lib, dtype=_native.TD_F32, B=1, Q=4, N=10, C=16, H=2, HD=16, L=2, P=2, ptr=1):
    err = _err()
    p = ctypes.c_void_p(ptr) if ptr else None
    rc = lib.td_fused_forward(dtype, p, p, None, p, p, p, p, p, B, Q, N, C, H, HD, L, P, None, err, 256)
    return rc, err.value.decode()


def test_argument_errors_return_before_any_launch(lib):
    assert call_fused(lib, L=8, P=9) == (1, 'levels x points must be <= 64')
    assert call_fused(lib, H=0)[0] == 1
    assert call_fused(lib, HD=15)[0] == 1
    assert call_fused(lib, C=9000)[1] == 'channels must be <= 8192'
    assert call_fused(lib, dtype=7)[0] == 1
    assert call_fused(lib, N=2 ** 31)[1] == 'too many memory tokens'
    assert call_fused(lib, B=2 ** 20, Q=2 ** 10, H=8)[1] == 'too many (batch, query, head) rows'
    assert call_fused(lib, ptr=0)[1] == 'null tensor pointer'


def test_empty_work_is_a_no_op(lib):
    assert call_fused(lib, Q=0, ptr=0) == (0, '')
    assert call_fused(lib, B=0, ptr=0) == (0, '')


def test_project_needs_a_big_enough_workspace(lib):
    err = _err()
    p = ctypes.c_void_p(16)
    rc = lib.td_project_forward(_native.TD_F16, p, p, None, p, p, p, p, p, 1, 4, 10, 16, 2, 16, 2, 2,
                                p, 10, None, err, 256)
    assert rc == 3 and 'workspace' in err.value.decode()
