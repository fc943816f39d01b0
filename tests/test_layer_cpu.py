"""The sampling producer and the whole deformable attention layer on CPU: the float64 oracle against the torch
restatement (Deformable-DETR's MSDeformAttn forward: offsets and logits from the query, softmax over L * P, 2-d
reference points or 4-d reference boxes), the CPU route of the public functions, weight packing and argument errors.
Upstream has no producer, so these pin the restatement against torch's operators, not against upstream."""

import numpy as np
import pytest
import torch

from cases import make_layer
from marearts_tinydeform_b200 import (deform_attn_layer, deform_attn_layer_reference, pack_sampling_weights,
                                      sampling_producer, sampling_producer_reference)
from oracle import deform_oracle as O

SMALL_LAYERS = [
    # name, B, Q, Cq, H, D, C, levels, P
    ('two levels', 2, 9, 32, 4, 8, 32, [(7, 9), (4, 5)], 4),
    ('four levels non-square', 1, 12, 64, 8, 8, 64, [(10, 15), (5, 8), (3, 4), (2, 2)], 4),
    ('max level points', 1, 5, 16, 2, 8, 16, [(6, 6), (3, 3), (2, 2), (1, 1)], 16),
    ('one point', 2, 4, 24, 3, 4, 12, [(5, 4)], 1),
    ('odd', 1, 7, 20, 3, 6, 18, [(5, 7), (3, 4), (2, 2)], 3),
]


def _producer_args(args, H, P):
    q, ref, _, shapes, _, sw, sb, _, _ = args
    return q, ref, shapes, H, P, sw, sb


@pytest.mark.parametrize('ref_dim', [2, 4])
@pytest.mark.parametrize('case', SMALL_LAYERS, ids=[c[0] for c in SMALL_LAYERS])
def test_oracle_producer_matches_torch(case, ref_dim):
    _, B, Q, Cq, H, D, C, levels, P = case
    for bias in (True, False):
        args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim, dtype=torch.float64, bias=bias, seed=Q)
        loc, attn = O.sampling_producer_oracle(*_producer_args(args, H, P))
        want_loc, want_attn = sampling_producer_reference(*_producer_args(args, H, P))
        assert loc.shape == (B, Q, H, len(levels), P, 2) and attn.shape == (B, Q, H, len(levels), P)
        np.testing.assert_allclose(loc, want_loc.numpy(), rtol=0, atol=1e-13)
        np.testing.assert_allclose(attn, want_attn.numpy(), rtol=0, atol=1e-15)
        np.testing.assert_allclose(attn.reshape(B, Q, H, -1).sum(-1), 1.0, atol=1e-13)


def test_producer_zero_offsets_land_on_the_reference_points():
    """Zero offset rows: every point of every head sits on its level's reference point (both forms), and equal
    logits give uniform weights 1 / (L * P)."""
    B, Q, Cq, H, D, C, levels, P = 1, 6, 16, 2, 8, 16, [(6, 6), (3, 3)], 4
    L = len(levels)
    for ref_dim in (2, 4):
        q, ref, _, shapes, _, sw, _, _, _ = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim,
                                                       dtype=torch.float64, seed=3)
        sw = sw.clone()
        sw[:2 * H * L * P] = 0
        sw[2 * H * L * P:] = 0
        loc, attn = O.sampling_producer_oracle(q, ref, shapes, H, P, sw, None)
        np.testing.assert_array_equal(loc, np.broadcast_to(ref[:, :, None, :, None, :2].numpy(), loc.shape))
        np.testing.assert_allclose(attn, 1.0 / (L * P), atol=1e-15)


def test_producer_from_proj_is_the_oracle_split():
    args = make_layer(2, 5, 16, 2, 8, 16, [(6, 6), (3, 3)], 4, ref_dim=4, dtype=torch.float64, seed=8)
    q, ref, _, shapes, _, sw, sb, _, _ = args
    loc, attn = O.sampling_producer_oracle(q, ref, shapes, 2, 4, sw, sb)
    loc2, attn2 = O.producer_from_proj(O.project(q, sw, sb), ref, shapes, 2, 4)
    np.testing.assert_array_equal(loc, loc2)
    np.testing.assert_array_equal(attn, attn2)


@pytest.mark.parametrize('ref_dim', [2, 4])
def test_oracle_layer_matches_torch(ref_dim):
    for i, (_, B, Q, Cq, H, D, C, levels, P) in enumerate(SMALL_LAYERS):
        args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim, dtype=torch.float64, seed=20 + i)
        N = args[2].shape[1]
        g = torch.Generator().manual_seed(i)
        mask = torch.rand(B, N, generator=g) < 0.3
        wo = torch.randn(11, H * D, generator=g, dtype=torch.float64) / (H * D) ** 0.5
        bo = torch.randn(11, generator=g, dtype=torch.float64) * 0.1
        for extra in ({}, {'value_padding_mask': mask}, {'output_weight': wo, 'output_bias': bo},
                      {'output_weight': wo, 'value_padding_mask': mask}):
            got = O.deform_attn_layer_oracle(*args[:5], H, P, *args[5:], **extra)
            want = deform_attn_layer_reference(*args[:5], H, P, *args[5:], **extra)
            np.testing.assert_allclose(got, want.numpy(), rtol=0, atol=1e-12, err_msg=f'{i} {sorted(extra)}')


def test_layer_cpu_route_is_the_reference():
    _, B, Q, Cq, H, D, C, levels, P = SMALL_LAYERS[1]
    for dtype in (torch.float32, torch.float64):
        args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=4, dtype=dtype, seed=5)
        for mode in ('auto', 'fused', 'project'):
            assert torch.equal(deform_attn_layer(*args[:5], H, P, *args[5:], mode=mode),
                               deform_attn_layer_reference(*args[:5], H, P, *args[5:]))
        loc, attn = sampling_producer(*_producer_args(args, H, P))
        want_loc, want_attn = sampling_producer_reference(*_producer_args(args, H, P))
        assert torch.equal(loc, want_loc) and torch.equal(attn, want_attn)


def test_pack_sampling_weights():
    g = torch.Generator().manual_seed(0)
    w_off, b_off = torch.randn(48, 16, generator=g), torch.randn(48, generator=g)
    w_att, b_att = torch.randn(24, 16, generator=g), torch.randn(24, generator=g)
    w, b = pack_sampling_weights(w_off, b_off, w_att, b_att)
    assert torch.equal(w, torch.cat([w_off, w_att])) and torch.equal(b, torch.cat([b_off, b_att]))
    assert pack_sampling_weights(w_off, None, w_att, None)[1] is None
    _, b = pack_sampling_weights(w_off, None, w_att, b_att)
    assert torch.equal(b[:48], torch.zeros(48)) and torch.equal(b[48:], b_att)
    # the packed projection is the two nn.Linear projections side by side
    x = torch.randn(3, 16, generator=g)
    w, b = pack_sampling_weights(w_off, b_off, w_att, b_att)
    torch.testing.assert_close(torch.nn.functional.linear(x, w, b),
                               torch.cat([torch.nn.functional.linear(x, w_off, b_off),
                                          torch.nn.functional.linear(x, w_att, b_att)], -1))


def test_layer_argument_errors():
    _, B, Q, Cq, H, D, C, levels, P = SMALL_LAYERS[0]
    args = make_layer(B, Q, Cq, H, D, C, levels, P, seed=1)
    with pytest.raises(ValueError):
        deform_attn_layer(*args[:5], H, P, *args[5:], mode='gather')
    with pytest.raises(ValueError):
        deform_attn_layer(*args[:5], H, P, *args[5:], output_bias=torch.zeros(4))
