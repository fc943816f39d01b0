"""The backward oracle is pinned: it reproduces the gradients that torch autograd gives through upstream's own
ma_deform_attn_reference (tests/golden/golden_grads.npz, written by tests/golden/make_golden_grads.py), and agrees
with central finite differences of the forward oracle. The public CPU route (ma_deform_attn on CPU tensors) is the
reference itself, with autograd."""

import json
import os

import numpy as np
import pytest
import torch

from cases import make
from marearts_tinydeform_b200 import ma_deform_attn
from oracle import deform_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden', 'golden_grads.npz')
NAMES = ('memory', 'value_weight', 'value_bias', 'spatial_shapes', 'level_start_index', 'sampling_locations',
         'attention_weights')
DTYPES = {'float32': torch.float32, 'float16': torch.float16, 'bfloat16': torch.bfloat16, 'float64': torch.float64}


def load_grads():
    z = np.load(GOLDEN)
    cases = []
    for entry in json.loads(bytes(z['manifest']).decode()):
        key = entry['key']
        inputs = []
        for field in NAMES:
            name = f'{key}/{field}'
            if name not in z:
                inputs.append(None)
                continue
            a = z[name]
            t = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16) if a.dtype == np.uint16 \
                else torch.from_numpy(a.copy())
            inputs.append(t)
        mask = torch.from_numpy(z[f'{key}/value_padding_mask'].astype(bool)) \
            if f'{key}/value_padding_mask' in z else None
        want = {g: z[f'{key}/grad_{g}'] for g in entry['grads']}
        cases.append((key, DTYPES[entry['dtype']], inputs, mask, torch.from_numpy(z[f'{key}/grad_out']), want))
    return cases


GRAD_CASES = load_grads()


def upcast(inputs):
    return [t if t is None or t.dtype == torch.long else t.double() for t in inputs]


def test_grad_fixture_is_complete():
    keys = {c[0] for c in GRAD_CASES}
    for must in ('tiny', 'far-outside', 'no-bias', 'max-level-points', 'boundary-locations', 'float64',
                 'masked-fp32', 'masked-bf16-one-image-padded'):
        assert must in keys
    assert all('sampling_locations' in c[5] and 'memory' in c[5] for c in GRAD_CASES)


@pytest.mark.parametrize('case', GRAD_CASES, ids=[c[0] for c in GRAD_CASES])
def test_backward_oracle_matches_upstream_autograd(case):
    key, _, inputs, mask, grad_out, want = case
    got = O.ma_deform_attn_backward_oracle(*upcast(inputs), grad_out, mask)
    for name, w in want.items():
        np.testing.assert_allclose(got[name], w, rtol=0, atol=1e-11 * max(1.0, float(np.abs(w).max())),
                                   err_msg=f'{key}: grad of {name}')
    if 'value_bias' not in want:
        assert got['value_bias'] is None


def test_backward_oracle_planted_mistake_is_caught():
    """Differentiating with dx/dloc = w / 2 (the grid-space derivative without the 2 loc - 1 chain factor) must
    fail against the golden vectors."""
    key, _, inputs, mask, grad_out, want = next(c for c in GRAD_CASES if c[0] == 'tiny')
    got = O.ma_deform_attn_backward_oracle(*upcast(inputs), grad_out, mask)
    wrong = got['sampling_locations'] / 2
    assert np.abs(wrong - want['sampling_locations']).max() > 1e-3


def test_backward_oracle_matches_finite_differences():
    args = make(1, 5, 2, 4, 8, [(5, 6), (3, 3)], 3, dtype=torch.float64, seed=9)
    g = torch.randn(1, 5, 8, generator=torch.Generator().manual_seed(2), dtype=torch.float64)
    grads = O.ma_deform_attn_backward_oracle(*args, g)

    def f(a):
        return float((O.ma_deform_attn_oracle(*a) * g.numpy()).sum())

    rng = np.random.default_rng(0)
    for idx, name in ((0, 'memory'), (1, 'value_weight'), (5, 'sampling_locations'), (6, 'attention_weights')):
        flat = args[idx].reshape(-1)
        for j in rng.choice(flat.numel(), 6, replace=False):
            eps = 1e-6
            plus = [t.clone() if t is not None else None for t in args]
            minus = [t.clone() if t is not None else None for t in args]
            plus[idx].view(-1)[j] += eps
            minus[idx].view(-1)[j] -= eps
            fd = (f(plus) - f(minus)) / (2 * eps)
            assert abs(fd - grads[name].reshape(-1)[j]) < 1e-6 * max(1.0, abs(fd)), f'{name}[{j}]'


def test_cpu_route_has_autograd():
    args = make(1, 6, 2, 8, 16, [(6, 7), (3, 4)], 2, dtype=torch.float64, seed=3)
    x = [t.clone().requires_grad_(True) if t is not None and t.dtype == torch.float64 else t for t in args]
    g = torch.randn(1, 6, 16, generator=torch.Generator().manual_seed(1), dtype=torch.float64)
    ma_deform_attn(*x).backward(g)
    want = O.ma_deform_attn_backward_oracle(*args, g)
    for i, name in ((0, 'memory'), (1, 'value_weight'), (2, 'value_bias'), (5, 'sampling_locations'),
                    (6, 'attention_weights')):
        np.testing.assert_allclose(x[i].grad.numpy(), want[name], rtol=0, atol=1e-12)
