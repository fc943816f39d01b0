"""The oracle is pinned: it must reproduce the golden vectors written by upstream's own ma_deform_attn_reference."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import deform_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden', 'golden_vectors.npz')
NAMES = ('memory', 'value_weight', 'value_bias', 'spatial_shapes', 'level_start_index', 'sampling_locations',
         'attention_weights')
DTYPES = {'float32': torch.float32, 'float16': torch.float16, 'bfloat16': torch.bfloat16, 'float64': torch.float64}


MASKS = {}  # key -> value padding mask (bool [B, N]) of the masked cases


def load_golden():
    z = np.load(GOLDEN)
    manifest = json.loads(bytes(z['manifest']).decode())
    cases = []
    for entry in manifest:
        key, dtype = entry['key'], DTYPES[entry['dtype']]
        inputs = []
        for field in NAMES:
            name = f'{key}/{field}'
            if name not in z:
                inputs.append(None)
                continue
            a = z[name]
            if a.dtype == np.uint16:
                t = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
            else:
                t = torch.from_numpy(a.copy())
            inputs.append(t)
        native = torch.from_numpy(z[f'{key}/expected_native']) if f'{key}/expected_native' in z else None
        if f'{key}/value_padding_mask' in z:
            MASKS[key] = torch.from_numpy(z[f'{key}/value_padding_mask'].astype(bool))
        cases.append((key, dtype, inputs, torch.from_numpy(z[f'{key}/expected_f64']), native))
    return cases


CASES = load_golden()
IDS = [c[0] for c in CASES]


def upcast(inputs):
    return [t if t is None or t.dtype == torch.long else t.double() for t in inputs]


def test_golden_fixture_is_complete():
    keys = {c[0] for c in CASES}
    assert len(CASES) >= 13
    for must in ('tiny', 'far-outside', 'no-bias', 'max-level-points', 'odd-channels', 'boundary-locations',
                 'narrow-heads-bf16', 'float64', 'masked-fp32', 'masked-fp16', 'masked-bf16-one-image-padded'):
        assert must in keys
    assert set(MASKS) == {'masked-fp32', 'masked-fp16', 'masked-bf16-one-image-padded'}
    for key, dtype, inputs, _, _ in CASES:
        assert inputs[0].dtype == dtype, key


@pytest.mark.parametrize('case', CASES, ids=IDS)
def test_numpy_oracle_matches_upstream(case):
    key, _, inputs, expected, _ = case
    got = O.ma_deform_attn_oracle(*inputs, value_padding_mask=MASKS.get(key))
    np.testing.assert_allclose(got, expected.numpy(), rtol=1e-12, atol=1e-12, err_msg=key)


@pytest.mark.parametrize('case', CASES, ids=IDS)
def test_fused_order_matches_upstream(case):
    key, _, inputs, expected, _ = case
    got = O.fused_order(*inputs, value_padding_mask=MASKS.get(key))
    np.testing.assert_allclose(got, expected.numpy(), rtol=1e-10, atol=1e-10, err_msg=key)


@pytest.mark.parametrize('case', CASES, ids=IDS)
def test_row_oracle_matches_upstream(case):
    key, _, inputs, expected, _ = case
    B, Q = expected.shape[:2]
    if Q == 0:
        return
    picks = [(b, q) for b in range(B) for q in range(0, Q, max(1, Q // 5))]
    got = O.oracle_rows(*inputs, picks, value_padding_mask=MASKS.get(key))
    want = np.stack([expected[b, q].numpy() for b, q in picks])
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-10, err_msg=key)


@pytest.mark.parametrize('case', CASES, ids=IDS)
def test_torch_port_matches_upstream(case):
    key, _, inputs, expected, native = case
    got = O.torch_port(*upcast(inputs), value_padding_mask=MASKS.get(key))
    torch.testing.assert_close(got, expected, rtol=1e-12, atol=1e-12, msg=key)
    if native is not None:  # same operators in float32: equal to upstream's float32 result up to rounding
        torch.testing.assert_close(O.torch_port(*inputs), native, rtol=1e-5, atol=1e-6, msg=key)


@pytest.mark.parametrize('case', CASES, ids=IDS)
def test_package_reference_matches_upstream(case):
    from marearts_tinydeform_b200 import ma_deform_attn_reference
    key, _, inputs, expected, native = case
    with torch.no_grad():
        got = ma_deform_attn_reference(*upcast(inputs), value_padding_mask=MASKS.get(key))
    torch.testing.assert_close(got, expected, rtol=1e-12, atol=1e-12, msg=key)
    if native is not None:
        with torch.no_grad():
            torch.testing.assert_close(ma_deform_attn_reference(*inputs), native, rtol=1e-5, atol=1e-6, msg=key)


def test_oracle_rejects_a_planted_mistake():
    """A wrong sampling rule (align_corners=True instead of False) must not pass the golden check."""
    key, _, inputs, expected, _ = CASES[0]
    saved = O.level_corners

    def align_corners_true(loc_xy, attn, height, width, start, n_tok):
        # pixel = loc * (size - 1): the align_corners=True mapping
        shifted = loc_xy.copy()
        shifted[..., 0] = (loc_xy[..., 0] * (width - 1) + 0.5) / width
        shifted[..., 1] = (loc_xy[..., 1] * (height - 1) + 0.5) / height
        return saved(shifted, attn, height, width, start, n_tok)

    O.level_corners = align_corners_true
    try:
        got = O.ma_deform_attn_oracle(*inputs)
    finally:
        O.level_corners = saved
    assert not np.allclose(got, expected.numpy(), rtol=1e-3, atol=1e-3)


def test_nan_and_inf_locations_sample_nothing():
    """Upstream's CUDA rule (csrc/ma_deform_fused.cu:87-89): NaN / inf locations contribute zero, finite far-away
    ones too; the oracle follows it."""
    tok, wt = O.level_corners(np.array([[np.nan, 0.5], [np.inf, 0.5], [-np.inf, 0.2], [1e30, 0.5]]),
                              np.ones(4), 4, 5, 0, 20)
    assert (tok == -1).all() and (wt == 0).all()
