"""The sampling producer and the whole layer against closed-form golden cases (tests/golden/producer_closed_form.npz,
written by tests/golden/make_producer_golden.py from Deformable-DETR's published definition by construction: zero
query weights, reference points on pixel centres and whole-pixel offsets, so every location is a pixel centre and the
output is indexing plus a softmax-weighted sum). Both reference forms (points and boxes); the torch restatement and
the oracle on the CPU, the layer kernels in both orders on the GPU."""

import os

import numpy as np
import pytest
import torch

from marearts_tinydeform_b200 import deform_attn_layer, deform_attn_layer_reference, sampling_producer_reference
from oracle import deform_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden', 'producer_closed_form.npz')


def load():
    z = np.load(GOLDEN)
    return {k: z[k] for k in z.files}


def layer_args(g, form, dtype=torch.float64, device='cpu'):
    f = lambda k: torch.from_numpy(g[k]).to(device=device, dtype=dtype)
    ref = f('ref2' if form == 2 else 'ref4')
    bias = f('sampling_bias2' if form == 2 else 'sampling_bias4')
    shapes = torch.from_numpy(g['spatial_shapes']).to(device)
    starts = torch.from_numpy(g['level_start_index']).to(device)
    return (f('query'), ref, f('memory'), shapes, starts, int(g['n_heads']), int(g['n_points']),
            f('sampling_weight'), bias, f('value_weight'), f('value_bias'))


def test_the_fixture_matches_its_generator():
    from golden.make_producer_golden import make
    g, fresh = load(), make()
    for k in fresh:
        assert np.array_equal(g[k], fresh[k]), k


@pytest.mark.parametrize('form', [2, 4])
def test_torch_restatement_and_oracle_match_the_closed_form(form):
    g = load()
    q, ref, mem, shapes, starts, H, P, sw, sb, vw, vb = layer_args(g, form)
    loc, attn = sampling_producer_reference(q, ref, shapes, H, P, sw, sb)
    np.testing.assert_allclose(loc.numpy(), g['locations'], atol=1e-12)
    np.testing.assert_allclose(attn.numpy(), g['weights'], atol=1e-12)
    out = deform_attn_layer_reference(q, ref, mem, shapes, starts, H, P, sw, sb, vw, vb)
    np.testing.assert_allclose(out.numpy(), g['out'], atol=1e-9)
    o_loc, o_attn = O.sampling_producer_oracle(q, ref, shapes, H, P, sw, sb)
    np.testing.assert_allclose(o_loc, g['locations'], atol=1e-12)
    np.testing.assert_allclose(o_attn, g['weights'], atol=1e-12)
    o_out = O.deform_attn_layer_oracle(q, ref, mem, shapes, starts, H, P, sw, sb, vw, vb)
    np.testing.assert_allclose(o_out, g['out'], atol=1e-9)


def test_a_planted_mistake_is_caught():
    """Offsets divided by (h, w) instead of (w, h): the closed form must reject it."""
    g = load()
    q, ref, mem, shapes, starts, H, P, sw, sb, vw, vb = layer_args(g, 2)
    swapped = torch.stack([shapes[:, 1], shapes[:, 0]], -1)
    loc, _ = sampling_producer_reference(q, ref, swapped, H, P, sw, sb)
    assert np.abs(loc.numpy() - g['locations']).max() > 1e-3


@pytest.mark.gpu
@pytest.mark.parametrize('form', [2, 4])
# 16-bit inputs move the reference points off the pixel centres by up to half an ulp (0.002 of a pixel in float16,
# 0.01 in bfloat16 at these map sizes), which mixes in that much of a neighbouring pixel's value
@pytest.mark.parametrize('dtype,tol', [(torch.float32, 2e-5), (torch.float16, 1e-2), (torch.bfloat16, 5e-2)])
def test_layer_kernels_match_the_closed_form(cuda, form, dtype, tol):
    g = load()
    args = layer_args(g, form, dtype=dtype, device=cuda)
    want = torch.from_numpy(g['out'])
    with torch.inference_mode():
        for mode in ('project', 'fused'):
            got = deform_attn_layer(*args, mode=mode).double().cpu()
            err = (got - want).abs().max().item()
            assert torch.allclose(got, want, atol=tol, rtol=tol), f'{dtype} form {form} [{mode}]: {err:.3g}'
