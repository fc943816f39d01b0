"""Parity of the sampling producer and the whole deformable attention layer on the GPU (through the C ABI):

  * the producer kernel (td_sampling_producer) against the float64 oracle fed with the same query projection, both
    reference forms, every dtype, L * P from 1 to 64;
  * the layer's fused order (td_layer_forward, TD_ORDER_FUSED) against its parts called one by one (projection,
    producer, ma_deform_attn 'fused', output projection): bit for bit;
  * the layer's project order, whose sampler computes the softmax and locations itself, against the float64 oracle
    fed with the GPU's query projection, at the same tolerances as the operator's parity tests, with and without the
    value padding mask and the output projection, on both kernel policies;
  * CUDA-graph capture, the 'auto' pick, empty query sets and rejected arguments."""

import numpy as np
import pytest
import torch

from cases import LAYER_CASES, make_layer
from marearts_tinydeform_b200 import _native, deform_attn_layer, ma_deform_attn, sampling_producer
from oracle import deform_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (3e-3, 3e-3), torch.bfloat16: (2e-2, 2e-2),
       torch.float64: (1e-12, 1e-10)}
# the producer's own outputs are rounded once to the dtype: half an ulp of values up to ~2
PRODUCER_TOL = {torch.float32: (2e-6, 2e-6), torch.float16: (1e-3, 1e-3), torch.bfloat16: (8e-3, 8e-3),
                torch.float64: (1e-13, 1e-12)}
DTYPES = (torch.float32, torch.float16, torch.bfloat16, torch.float64)


def _cuda(ts):
    return [None if t is None else t.cuda() for t in ts]


def _f64(t):
    return None if t is None or t.dtype == torch.long else t.double().cpu()


def _extras(case_index, B, N, HD, dtype):
    """(mask, output_weight, output_bias) variants of a case."""
    g = torch.Generator().manual_seed(100 + case_index)
    mask = torch.rand(B, N, generator=g) < 0.3
    wo = ((torch.rand(96, HD, generator=g) * 2 - 1) / HD ** 0.5).to(dtype)
    bo = ((torch.rand(96, generator=g) * 2 - 1) * 0.05).to(dtype)
    return [(None, None, None), (mask, None, None), (None, wo, bo), (mask, wo, None)]


@pytest.mark.parametrize('dtype', DTYPES)
@pytest.mark.parametrize('ref_dim', [2, 4])
def test_producer_kernel(cuda, dtype, ref_dim):
    for i, (name, B, Q, Cq, H, D, C, levels, P) in enumerate(LAYER_CASES):
        args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim, dtype=dtype, seed=i)
        q, ref, _, shapes, _, sw, sb, _, _ = _cuda(args)
        with torch.inference_mode():
            proj = _native.linear(q, sw, sb)
            loc, attn = _native.sampling_producer(proj, ref, shapes, H, P)
        want_loc, want_attn = O.producer_from_proj(proj.double().cpu(), _f64(args[1]), args[3], H, P)
        atol, rtol = PRODUCER_TOL[dtype]
        np.testing.assert_allclose(loc.double().cpu().numpy(), want_loc, atol=atol, rtol=rtol,
                                   err_msg=f'{name} {dtype} ref_dim={ref_dim}: locations')
        np.testing.assert_allclose(attn.double().cpu().numpy(), want_attn, atol=atol, rtol=rtol,
                                   err_msg=f'{name} {dtype} ref_dim={ref_dim}: weights')


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_layer_fused_order_is_its_parts(policy, dtype):
    for i, (name, B, Q, Cq, H, D, C, levels, P) in enumerate(LAYER_CASES):
        for ref_dim in (2, 4):
            args = _cuda(make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim, dtype=dtype, seed=10 + i))
            q, ref, mem, shapes, starts, sw, sb, vw, vb = args
            for mask, wo, bo in _extras(i, B, mem.shape[1], H * D, dtype):
                mask, wo, bo = _cuda([mask, wo, bo])
                with torch.inference_mode():
                    got = _native.layer_forward(q, ref, mem, shapes, starts, H, P, sw, sb, vw, vb, wo, bo, mask,
                                                order='fused')
                    loc, attn = sampling_producer(q, ref, shapes, H, P, sw, sb)
                    want = ma_deform_attn(mem, vw, vb, shapes, starts, loc, attn, mode='fused',
                                          value_padding_mask=mask)
                    if wo is not None:
                        want = _native.linear(want, wo, bo)
                assert torch.equal(got, want), f'{name} {dtype} ref_dim={ref_dim} mask={mask is not None} ' \
                                               f'out_proj={wo is not None} {policy}'


def _oracle_layer(args, proj, H, P, mask, wo, bo):
    """float64 layer from the GPU's query projection: producer, operator, output projection."""
    _, ref, mem, shapes, starts, _, _, vw, vb = args
    loc, attn = O.producer_from_proj(proj.double().cpu(), _f64(ref), shapes, H, P)
    out = O.ma_deform_attn_oracle(_f64(mem), _f64(vw), _f64(vb), shapes, starts, loc, attn,
                                  None if mask is None else mask.cpu())
    return out if wo is None else O.project(out, _f64(wo), _f64(bo))


@pytest.mark.parametrize('dtype', DTYPES)
def test_layer_project_order(policy, dtype):
    if dtype == torch.float64 and policy == 'cuda-cores':
        pytest.skip('float64 runs on CUDA cores under both policies')
    for i, (name, B, Q, Cq, H, D, C, levels, P) in enumerate(LAYER_CASES):
        ref_dim = 2 + 2 * (i % 2)
        args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim, dtype=dtype, seed=30 + i)
        dev = _cuda(args)
        q, ref, mem, shapes, starts, sw, sb, vw, vb = dev
        with torch.inference_mode():
            proj = _native.linear(q, sw, sb)
        for mask, wo, bo in _extras(i, B, mem.shape[1], H * D, dtype):
            want = torch.from_numpy(_oracle_layer(args, proj, H, P, mask, wo, bo))
            mask_d, wo_d, bo_d = _cuda([mask, wo, bo])
            with torch.inference_mode():
                got = _native.layer_forward(q, ref, mem, shapes, starts, H, P, sw, sb, vw, vb, wo_d, bo_d, mask_d,
                                            order='project').double().cpu()
            atol, rtol = TOL[dtype]
            err = (got - want).abs().max().item()
            assert torch.allclose(got, want, atol=atol, rtol=rtol), \
                f'{name} {dtype} ref_dim={ref_dim} mask={mask is not None} out_proj={wo is not None} {policy}: ' \
                f'max |diff| {err:.3g}'


def test_layer_orders_agree_and_auto(cuda):
    """Both orders give the same layer output in float32 (in float16 the fused order's locations are rounded to
    float16: half an ulp near 1 is 0.02 pixel at 80 pixels wide, enough to move single outputs of unit-variance random
    memory by several 1e-2, so there each order is checked against the oracle on its own, above); 'auto' is one of
    the two orders bit for bit."""
    for i, (name, B, Q, Cq, H, D, C, levels, P) in enumerate(LAYER_CASES[:3]):
        for dtype in (torch.float32, torch.float16):
            args = _cuda(make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=4, dtype=dtype, seed=50 + i))
            with torch.inference_mode():
                outs = {m: deform_attn_layer(*args[:5], H, P, *args[5:], mode=m)
                        for m in ('fused', 'project', 'auto')}
            if dtype == torch.float32:
                err = (outs['fused'] - outs['project']).abs().max().item()
                assert torch.allclose(outs['fused'], outs['project'], atol=1e-4, rtol=1e-4), f'{name}: {err:.3g}'
            assert torch.equal(outs['auto'], outs['fused']) or torch.equal(outs['auto'], outs['project']), name


def test_layer_in_a_cuda_graph(cuda):
    name, B, Q, Cq, H, D, C, levels, P = LAYER_CASES[0]
    args = _cuda(make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=2, dtype=torch.float16, seed=61))
    wo = torch.randn(256, H * D, device='cuda', dtype=torch.float16) / (H * D) ** 0.5
    with torch.inference_mode():
        eager = {m: deform_attn_layer(*args[:5], H, P, *args[5:], output_weight=wo, mode=m)
                 for m in ('fused', 'project')}
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for m in ('fused', 'project'):
                deform_attn_layer(*args[:5], H, P, *args[5:], output_weight=wo, mode=m)
        torch.cuda.current_stream().wait_stream(side)
        for m in ('fused', 'project'):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = deform_attn_layer(*args[:5], H, P, *args[5:], output_weight=wo, mode=m)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, eager[m]), m


def test_layer_empty_queries_and_errors(cuda):
    name, B, Q, Cq, H, D, C, levels, P = LAYER_CASES[2]
    args = _cuda(make_layer(B, Q, Cq, H, D, C, levels, P, dtype=torch.float32, seed=70))
    q, ref, mem, shapes, starts, sw, sb, vw, vb = args
    with torch.inference_mode():
        empty = deform_attn_layer(q[:, :0], ref[:, :0], mem, shapes, starts, H, P, sw, sb, vw, vb)
        assert empty.shape == (B, 0, H * D)
        bad = [
            dict(sampling_weight=sw[:-1]),                                    # not 3 * H * L * P rows
            dict(reference_points=ref[..., :1].expand(*ref.shape[:3], 3)),    # 3 coordinates
            dict(query=q.half()),                                             # dtype mismatch
            dict(value_padding_mask=torch.zeros(B, mem.shape[1] + 1, dtype=torch.bool, device='cuda')),
        ]
        base = dict(query=q, reference_points=ref, memory=mem, spatial_shapes=shapes, level_start_index=starts,
                    n_heads=H, n_points=P, sampling_weight=sw, sampling_bias=sb, value_weight=vw, value_bias=vb)
        for change in bad:
            with pytest.raises(RuntimeError):
                deform_attn_layer(**{**base, **change})
