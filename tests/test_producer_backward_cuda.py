"""Backward of the sampling producer on this library's kernels (td_sampling_producer_backward behind
autograd.ProducerFunction, the query projection behind LinearFunction). Checked against torch autograd of
sampling_producer_reference (the producer's definition: Deformable-DETR's MSDeformAttn forward, whose parity is
pinned by the closed-form golden cases) in float64 and in the kernels' own dtypes, for reference points and
reference boxes, with one output's gradient absent, by gradcheck in float64, and through a training step of the
whole layer that launches only this library's GEMMs."""

import numpy as np
import pytest
import torch

from cases import LAYER_CASES, make_layer
from marearts_tinydeform_b200 import _native, deform_attn_layer, sampling_producer, sampling_producer_reference
from marearts_tinydeform_b200.autograd import ProducerFunction

pytestmark = pytest.mark.gpu

# relative to the largest gradient of the tensor (a gradient that is zero everywhere must come out zero)
TOL = {torch.float64: 1e-10, torch.float32: 1e-5, torch.float16: 4e-3, torch.bfloat16: 3e-2}


def _close(got, want, tol, what):
    got = got.double().cpu()
    # autograd leaves the gradient of an input the loss does not reach as None: zero
    want = torch.zeros_like(got) if want is None else want.double().cpu()
    scale = max(float(want.abs().max()), 1e-30)
    err = float((got - want).abs().max()) / scale
    assert err <= tol, f'{what}: max |diff| / max |want| = {err:.3g} > {tol}'


def _grads(fn, query, ref, sw, sb, shapes, H, P, g_loc, g_attn):
    x = [t.detach().clone().requires_grad_(True) for t in (query, ref, sw, sb)]
    loc, attn = fn(x[0], x[1], shapes, H, P, x[2], x[3])
    terms = []
    if g_loc is not None:
        terms.append((loc * g_loc).sum())
    if g_attn is not None:
        terms.append((attn * g_attn).sum())
    sum(terms).backward()
    return (loc.detach(), attn.detach()), [t.grad for t in x]


@pytest.mark.parametrize('dtype', [torch.float64, torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize('ref_dim', [2, 4])
def test_producer_gradients_against_torch_autograd(cuda, dtype, ref_dim):
    names = ('query', 'reference points', 'sampling weight', 'sampling bias')
    for i, (name, B, Q, Cq, H, D, C, levels, P) in enumerate(LAYER_CASES):
        q, ref, _, shapes, _, sw, sb, _, _ = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim, dtype=dtype,
                                                        seed=700 + i)
        L = len(levels)
        g = torch.Generator().manual_seed(800 + i)
        g_loc = torch.randn(B, Q, H, L, P, 2, generator=g).to(dtype)
        g_attn = torch.randn(B, Q, H, L, P, generator=g).to(dtype)
        for which in ('both', 'loc', 'attn'):
            gl = g_loc if which != 'attn' else None
            ga = g_attn if which != 'loc' else None
            # the reference in float64 on the CPU, from the same (rounded) inputs
            _, want = _grads(sampling_producer_reference, q.double(), ref.double(), sw.double(), sb.double(),
                             shapes, H, P, None if gl is None else gl.double(), None if ga is None else ga.double())
            _, got = _grads(sampling_producer, q.cuda(), ref.cuda(), sw.cuda(), sb.cuda(), shapes.cuda(), H, P,
                            None if gl is None else gl.cuda(), None if ga is None else ga.cuda())
            for k in range(4):
                _close(got[k], want[k], TOL[dtype], f'{name} {dtype} ref_dim={ref_dim} grads of {which}: {names[k]}')


@pytest.mark.parametrize('ref_dim', [2, 4])
def test_producer_gradcheck_float64(cuda, ref_dim):
    name, B, Q, Cq, H, D, C, levels, P = LAYER_CASES[3]  # 16 level-points per head, four levels
    q, ref, _, shapes, _, sw, sb, _, _ = make_layer(1, 3, Cq, H, D, C, levels, P, ref_dim=ref_dim,
                                                    dtype=torch.float64, seed=900)
    proj = torch.nn.functional.linear(q, sw, sb).cuda().requires_grad_(True)
    r = ref.cuda().requires_grad_(True)
    shp = shapes.cuda()
    assert torch.autograd.gradcheck(lambda p, rr: ProducerFunction.apply(p, rr, shp, H, P), (proj, r),
                                    eps=1e-6, atol=1e-7, rtol=1e-5)


def test_layer_training_step_runs_only_library_gemms(cuda):
    """A training step of the whole layer (producer, attention, output_proj): every GEMM of the forward and the
    backward is this library's, and the producer's backward kernel runs."""
    name, B, Q, Cq, H, D, C, levels, P = LAYER_CASES[0]
    args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=4, dtype=torch.float16, seed=910)
    x = [t.cuda().requires_grad_(True) if t.is_floating_point() else t.cuda() for t in args]
    wo = (torch.randn(256, H * D, device='cuda') / 16).half().requires_grad_(True)
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        out = deform_attn_layer(*x[:5], H, P, *x[5:], output_weight=wo, mode='project')
        out.float().square().sum().backward()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    gemm_like = [n for n in names if any(k in n.lower() for k in ('gemm', 'cublas', 'cutlass', 'sm90_', 'sm100_',
                                                                  'nvjet', 'xmma')) and 'grad_gemm' not in n]
    assert not gemm_like, f'library GEMMs in the layer step: {sorted(set(gemm_like))}'
    assert any('sampling_producer_backward_kernel' in n for n in names), sorted(set(names))
    for t in x:
        if t.is_floating_point():
            assert t.grad is not None and torch.isfinite(t.grad.float()).all()
    assert _native.device_error() == 0


def test_producer_backward_rejects_bad_arguments(cuda):
    proj = torch.zeros(1, 2, 3 * 2 * 1 * 4, device='cuda')
    ref = torch.zeros(1, 2, 1, 3, device='cuda')
    shapes = torch.tensor([[4, 4]], device='cuda')
    with pytest.raises(RuntimeError, match='2 \\(x, y\\) or 4'):
        _native.sampling_producer_backward(proj, ref, shapes, 2, 4, None, None)
    # no incoming gradient at all: zeros
    ref2 = torch.rand(1, 2, 1, 2, device='cuda')
    gp, gr = _native.sampling_producer_backward(proj, ref2, shapes, 2, 4, None, None)
    assert float(gp.abs().max()) == 0.0 and float(gr.abs().max()) == 0.0
    assert np.isfinite(gp.cpu().numpy()).all()
