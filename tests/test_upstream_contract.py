"""Upstream's own test suite (tests/test_correctness.py, eight tests), restated against the drop-in import name.

Every check below is one of upstream's, with its shapes, seeds, tolerances and expectations, run against
``import marearts_tinydeform`` exactly as upstream's file imports it: the three CUDA paths ('fused', 'project',
'auto') against ``ma_deform_attn_reference``, float32 with TF32 off (atol 2e-5 / rtol 1e-4), float16 / bfloat16
against the reference in float64 (3e-3 / 2e-2), misaligned memory, far-outside and empty inputs, rejected inputs
(the inference-only rule among them), and the auto picker. The input recipe and the shape cases are upstream's
(tests/test_correctness.py:13-43), from tests/cases.py. The tests that need a GPU are marked ``gpu``; upstream's
versions of them return early without CUDA.
"""

import pytest
import torch

import marearts_tinydeform
from cases import CASES, make, to
from marearts_tinydeform import choose_mode, ma_deform_attn, ma_deform_attn_reference


def check(name, args, ref_args, atol, rtol):
    """Every mode of the drop-in against the reference on ref_args (tests/test_correctness.py:46-53)."""
    with torch.inference_mode():
        ref = ma_deform_attn_reference(*ref_args).float().cpu()
        for mode in ('fused', 'project', 'auto'):
            got = ma_deform_attn(*args, mode=mode).float().cpu()
            err = (got - ref).abs().max().item() if got.numel() else 0.0
            assert torch.allclose(got, ref, atol=atol, rtol=rtol), \
                f'{name} [{mode}]: max |diff| {err:.3g} (max |ref| {ref.abs().max().item():.3g})'


def _double(args):
    return [t if t is None or t.dtype == torch.long else t.double() for t in args]


def test_cpu_path_is_reference():
    args = make(1, 10, 2, 8, 16, [(6, 7), (3, 4)], 2)
    with torch.inference_mode():
        assert torch.equal(ma_deform_attn(*args), ma_deform_attn_reference(*args))


@pytest.mark.gpu
def test_cuda_float32(cuda):
    # the reference runs on the same CUDA tensors, with TF32 off (the cuda fixture turns it off)
    for name, *shape in CASES:
        for bias in (True, False):
            args = to(make(*shape, bias=bias), cuda)
            check(f'{name} fp32 bias={bias}', args, args, atol=2e-5, rtol=1e-4)


@pytest.mark.gpu
def test_cuda_half_and_bfloat16(cuda):
    for dtype, atol in ((torch.float16, 3e-3), (torch.bfloat16, 2e-2)):
        for name, *shape in CASES:
            args = make(*shape, dtype=dtype)
            check(f'{name} {dtype}', to(args, cuda), _double(args), atol=atol, rtol=atol)


@pytest.mark.gpu
def test_unaligned_memory_uses_scalar_kernel(cuda):
    for dtype, atol in ((torch.float32, 2e-5), (torch.float16, 3e-3)):
        args = make(1, 40, 8, 32, 256, [(20, 20), (10, 10)], 4, dtype=dtype)
        mem = args[0].to(cuda)
        buf = torch.empty(mem.numel() + 1, dtype=dtype, device=cuda)
        shifted = buf[1:].view(mem.shape)  # contiguous, 2 or 4 bytes off a 16-byte boundary
        shifted.copy_(mem)
        assert shifted.is_contiguous() and shifted.data_ptr() % 16 != 0
        dev = to(args, cuda)
        check(f'unaligned {dtype}', [shifted] + dev[1:], _double(args), atol=atol, rtol=atol)


@pytest.mark.gpu
def test_far_outside_and_empty(cuda):
    args = to(make(2, 20, 4, 8, 32, [(9, 11), (5, 6)], 4, spread=200.0), cuda)  # nearly every sample outside
    check('far outside', args, args, atol=1e-5, rtol=1e-4)
    empty = to(make(1, 0, 4, 8, 32, [(9, 11)], 4), cuda)
    with torch.inference_mode():
        for mode in ('fused', 'project'):
            assert ma_deform_attn(*empty, mode=mode).shape == (1, 0, 32)


@pytest.mark.gpu
def test_rejects_bad_input(cuda):
    args = to(make(1, 8, 2, 8, 16, [(6, 7), (3, 4)], 2), cuda)
    bad = [
        ('weight cols', 1, args[1][:, :8].contiguous()),
        ('dtype', 1, args[1].half()),
        ('bias size', 2, args[2][:4]),
        ('shapes dtype', 3, args[3].int()),
        ('too many points', 6, torch.ones(1, 8, 2, 2, 40, device=cuda) / 80),
    ]
    for what, i, value in bad:
        a = list(args)
        a[i] = value
        if what == 'too many points':
            a[5] = torch.rand(1, 8, 2, 2, 40, 2, device=cuda)
        for mode in ('fused', 'project'):  # the project order checks the weights itself, so no case is skipped
            with pytest.raises(RuntimeError):
                with torch.inference_mode():
                    ma_deform_attn(*a, mode=mode)
    grad = [t.clone().requires_grad_(True) if i == 0 else t for i, t in enumerate(args)]
    with pytest.raises(RuntimeError, match='inference only'):
        ma_deform_attn(*grad)
    with pytest.raises(ValueError):
        ma_deform_attn(*args, mode='nope')


def test_auto_picks_fused_for_few_queries():
    few = make(1, 50, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4)
    many = make(8, 900, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4)
    assert choose_mode(few[0], few[1], few[5]) == 'fused'
    assert choose_mode(many[0], many[1], many[5]) == 'project'


def test_auto_limits_follow_the_gpu_generation():
    get = torch.cuda.get_device_capability
    try:
        for cap, table in (((8, 9), marearts_tinydeform.FUSED_LIMIT),
                           ((7, 5), marearts_tinydeform.FUSED_LIMIT_SM75)):
            torch.cuda.get_device_capability = lambda device=None, cap=cap: cap
            assert marearts_tinydeform._limits.__wrapped__(0) is table
    finally:
        torch.cuda.get_device_capability = get
