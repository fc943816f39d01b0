"""Write tests/golden/golden_grads.npz: gradients of upstream's own ma_deform_attn_reference, by torch autograd.

Run once, in a checkout that has upstream MareArts/marearts-tinydeform v0.1.1 importable:

    python tests/golden/make_golden_grads.py --upstream <path to the upstream checkout>

Upstream's CUDA operator is inference only (it rejects inputs that require grad), but its reference
(marearts_tinydeform/reference.py:13-40: nn.Linear, grid_sample, weighted sum) is differentiable; these vectors are
what autograd gives through it, in float64 on the upcast inputs, for a seeded grad_out: the gradients with respect
to memory, value_weight, value_bias, sampling_locations and attention_weights. They pin the backward oracle
(tests/test_backward_cpu.py) and, through it, the backward kernels.

Masked cases (the mask is an addition; upstream has none): bias-free inputs, and upstream's reference run on
memory.masked_fill(mask, 0) inside the autograd graph -- the same function, and so the same gradients, as zeroing
the padded tokens' projected value.
"""

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from cases import SMALL_CASES, boundary_case, make, upcast  # noqa: E402
from make_golden import MASKED_CASES, NAMES, masked_case, to_numpy  # noqa: E402

GRAD_OF = {0: 'memory', 1: 'value_weight', 2: 'value_bias', 5: 'sampling_locations', 6: 'attention_weights'}
KEEP = ('tiny', 'rtdetr-mini', 'narrow-heads-bf16', 'one-level-many-points', 'odd-channels', 'far-outside',
        'no-bias', 'max-level-points', 'float64')


def grads(reference, inputs, grad_out, mask=None):
    x = [t if t is None or t.dtype == torch.long else t.detach().double().clone().requires_grad_(True)
         for t in inputs]
    mem = x[0] if mask is None else x[0].masked_fill(mask[..., None], 0)
    out = reference(mem, *x[1:])
    out.backward(grad_out)
    return {name: x[i].grad for i, name in GRAD_OF.items() if x[i] is not None}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--upstream', default=os.environ.get('TINYDEFORM_UPSTREAM', ''))
    ap.add_argument('--out', default=os.path.join(HERE, 'golden_grads.npz'))
    args = ap.parse_args()
    if not args.upstream:
        sys.exit('give --upstream <path to the upstream checkout>')
    sys.path.insert(0, args.upstream)
    from marearts_tinydeform.reference import ma_deform_attn_reference as upstream_reference

    cases = [(name, make(B, Q, H, D, C, levels, P, dtype=dtype, spread=spread, bias=bias, seed=i), dtype, None)
             for i, (name, B, Q, H, D, C, levels, P, dtype, spread, bias) in enumerate(SMALL_CASES) if name in KEEP]
    cases.append(('boundary-locations', boundary_case(), torch.float32, None))
    for i, (name, B, Q, H, D, C, levels, P, dtype, frac, whole) in enumerate(MASKED_CASES):
        inputs, mask = masked_case(i, B, Q, H, D, C, levels, P, dtype, frac, whole)
        cases.append((name, inputs, dtype, mask))
    arrays, manifest = {}, []
    for j, (name, inputs, dtype, mask) in enumerate(cases):
        key = name.replace(' ', '_')
        B, Q = inputs[5].shape[:2]
        HD = inputs[1].shape[0]
        grad_out = torch.randn(B, Q, HD, generator=torch.Generator().manual_seed(300 + j), dtype=torch.float64)
        g = grads(upstream_reference, upcast(inputs), grad_out, mask)
        for field, t in zip(NAMES, inputs):
            if t is not None:
                arrays[f'{key}/{field}'] = to_numpy(t)
        if mask is not None:
            arrays[f'{key}/value_padding_mask'] = mask.numpy().astype(np.uint8)
        arrays[f'{key}/grad_out'] = grad_out.numpy()
        for gname, t in g.items():
            arrays[f'{key}/grad_{gname}'] = t.numpy()
        manifest.append({'key': key, 'dtype': str(dtype).replace('torch.', ''), 'masked': mask is not None,
                         'grads': sorted(g)})
    arrays['manifest'] = np.frombuffer(json.dumps(manifest).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **arrays)
    print(f'wrote {len(manifest)} cases to {args.out} ({os.path.getsize(args.out)} bytes)')


if __name__ == '__main__':
    main()
