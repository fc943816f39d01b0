"""The project order's sampler with two rows a warp (sample_vec_kernel's kRW = 2: the corner prologue of both rows in
one pass, 16 lanes a row), which the library takes when the halved grid still gives every SM a CTA (at least 16 rows
per SM) and a row's points fit 16 lanes. Checked against the float64 oracle in every dtype, over the RT-DETR and DINO
geometries, an odd row count (the last warp's second row past the end), 9 points a row (lanes without a point),
16 points a row (every lane), 128- and 256-byte value rows, locations far outside the maps, a value padding mask and
the layer's project order (the producer's softmax over each row's 16 lanes); and against the same images run one at
a time, which take the one-wave forms (one row a warp, or two at another corner batch depth): the sums run in
different orders, so they agree to one unit in the last place."""

import pytest
import torch

from cases import make, make_layer, to, upcast
from marearts_tinydeform_b200 import _native, ma_deform_attn
from oracle import deform_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (2e-5, 1e-4), torch.float16: (3e-3, 3e-3), torch.bfloat16: (2e-2, 2e-2),
       torch.float64: (1e-10, 1e-10)}
ULP = {torch.float32: 2.0 ** -21, torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7, torch.float64: 2.0 ** -50}

# (name, B, Q, H, D, C, levels, P, spread); Q is raised where needed so that B * Q * H exceeds one wave
CASES = [
    ('rtdetr-640 b8', 8, 300, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4, 1.0),
    ('dino b2', 2, 900, 8, 32, 256, [(100, 167), (50, 84), (25, 42), (13, 21)], 4, 1.0),
    ('odd rows, 9 points', 3, 600, 3, 32, 96, [(12, 13), (6, 7), (3, 4)], 3, 1.0),
    ('16 points, 64-channel heads', 2, 400, 8, 64, 512, [(20, 20), (10, 10)], 8, 1.0),
    ('far outside the maps', 4, 200, 8, 32, 256, [(20, 24), (10, 12)], 4, 4.0),
]


def _rows_per_wave():
    return torch.cuda.get_device_properties(0).multi_processor_count * 40


def _close_ulp(a, b, dtype):
    """One unit in the last place of the larger, plus the accumulator's rounding over a row's 64 corner terms of
    magnitude up to ~4 (what two summation orders of a cancelling sum can differ by before the final rounding)."""
    acc_eps = 2.0 ** -53 if dtype == torch.float64 else 2.0 ** -24
    a, b = a.double(), b.double()
    return bool(((a - b).abs() <= ULP[dtype] * torch.maximum(a.abs(), b.abs()) + 256 * acc_eps).all())


@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16, torch.float32, torch.float64])
def test_two_rows_a_warp_against_oracle_and_one_row_form(cuda, dtype):
    wave = _rows_per_wave()
    for i, (name, B, Q, H, D, C, levels, P, spread) in enumerate(CASES):
        if dtype == torch.float64 and D == 64:
            continue  # 512-byte float64 rows would take 32 lanes a row: the one-row form
        Q = max(Q, wave // (B * H) + 1)
        if name.startswith('odd'):
            Q += (B * Q * H + 1) % 2  # an odd row count
            assert B * Q * H % 2 == 1
        assert B * Q * H > wave
        args = make(B, Q, H, D, C, levels, P, dtype=dtype, spread=spread, seed=800 + i)
        dev = to(args, 'cuda')
        with torch.inference_mode():
            got = ma_deform_attn(*dev, mode='project')
        want = torch.from_numpy(O.ma_deform_attn_oracle(*upcast(args)))
        atol, rtol = TOL[dtype]
        err = (got.double().cpu() - want).abs().max().item()
        assert torch.allclose(got.double().cpu(), want, atol=atol, rtol=rtol), f'{name} {dtype}: max |diff| {err:.3g}'
        if Q * H <= wave:  # one image is one wave
            for b in range(B):
                one = [dev[0][b:b + 1], *dev[1:5], dev[5][b:b + 1], dev[6][b:b + 1]]
                with torch.inference_mode():
                    single = ma_deform_attn(*one, mode='project')
                assert _close_ulp(got[b:b + 1], single, dtype), f'{name} {dtype} image {b}'


def test_two_rows_a_warp_with_padding_mask(cuda):
    B, H, D, C, levels, P = 4, 8, 32, 256, [(40, 40), (20, 20), (10, 10)], 4
    Q = max(200, _rows_per_wave() // (B * H) + 1)
    N = sum(h * w for h, w in levels)
    for dtype in (torch.float16, torch.bfloat16, torch.float32):
        args = make(B, Q, H, D, C, levels, P, dtype=dtype, seed=820)
        mask = torch.rand(B, N, generator=torch.Generator().manual_seed(821)) < 0.3
        with torch.inference_mode():
            got = ma_deform_attn(*to(args, 'cuda'), mode='project', value_padding_mask=mask.cuda())
        want = torch.from_numpy(O.ma_deform_attn_oracle(*upcast(args), value_padding_mask=mask.numpy()))
        atol, rtol = TOL[dtype]
        assert torch.allclose(got.double().cpu(), want, atol=atol, rtol=rtol), dtype


@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16, torch.float32])
def test_two_rows_a_warp_in_the_layer(cuda, dtype):
    """The layer's project order over several waves: the sampler's prologue runs the producer on each half-warp's row
    (reference points and boxes, an odd row count, a padding mask), against the float64 oracle layer built from the
    same query projection."""
    wave = _rows_per_wave()
    cases = [  # (B, Q, Cq, H, D, C, levels, P, ref_dim, mask)
        (4, 300, 256, 8, 32, 256, [(40, 40), (20, 20), (10, 10)], 4, 2, False),
        (4, 300, 256, 8, 32, 256, [(40, 40), (20, 20), (10, 10)], 4, 4, True),
        (3, 600, 96, 3, 32, 96, [(12, 13), (6, 7), (3, 4)], 3, 4, False),
    ]
    for i, (B, Q, Cq, H, D, C, levels, P, ref_dim, with_mask) in enumerate(cases):
        Q = max(Q, wave // (B * H) + 1)
        if H % 2:
            Q += (B * Q * H + 1) % 2  # an odd row count
        assert B * Q * H > wave
        args = make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=ref_dim, dtype=dtype, seed=840 + i)
        q, ref, mem, shapes, starts, sw, sb, vw, vb = [None if t is None else t.cuda() for t in args]
        N = sum(h * w for h, w in levels)
        mask = (torch.rand(B, N, generator=torch.Generator().manual_seed(850 + i)) < 0.3) if with_mask else None
        with torch.inference_mode():
            got = _native.layer_forward(q, ref, mem, shapes, starts, H, P, sw, sb, vw, vb, None, None,
                                        None if mask is None else mask.cuda(), order='project').double().cpu()
            proj = _native.linear(q, sw, sb)
        f64 = [None if t is None or t.dtype == torch.long else t.double() for t in args]
        loc, attn = O.producer_from_proj(proj.double().cpu(), f64[1], args[3], H, P)
        want = torch.from_numpy(O.ma_deform_attn_oracle(f64[2], f64[7], f64[8], args[3], args[4], loc, attn,
                                                        None if mask is None else mask.numpy()))
        atol, rtol = TOL[dtype]
        assert torch.allclose(got, want, atol=atol, rtol=rtol), \
            f'case {i} {dtype}: max |diff| {(got - want).abs().max().item():.3g}'
    assert _native.device_error(clear=True) == 0
