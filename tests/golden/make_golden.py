"""Write tests/golden/golden_vectors.npz from upstream's own ma_deform_attn_reference.

Run once, in a checkout that has upstream MareArts/marearts-tinydeform v0.1.1 importable (its path is given with
--upstream, default the environment variable TINYDEFORM_UPSTREAM):

    python tests/golden/make_golden.py --upstream <path to the upstream checkout>

For every case of tests/cases.py SMALL_CASES (plus the boundary-location case) it stores the inputs in their own
dtype and upstream's result computed in float64 on the upcast inputs, as upstream's tests do for float16 / bfloat16
(tests/test_correctness.py:79). bfloat16 arrays are stored as their uint16 bit patterns. The fixture is small
(a few MB) and is what pins the oracle: tests/test_oracle_golden.py checks the oracle against it.

Masked cases (the value padding mask is an addition; upstream has none): inputs without bias plus a bool mask
[B, N]; the expected result is upstream's reference run on memory with the padded rows zeroed, which is what
zeroing those tokens' projected value means when there is no bias.
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

NAMES = ('memory', 'value_weight', 'value_bias', 'spatial_shapes', 'level_start_index', 'sampling_locations',
         'attention_weights')

# name, B, Q, H, D, C, levels, P, dtype, padded fraction, images padded whole
MASKED_CASES = [
    ('masked-fp32', 2, 12, 8, 32, 256, [(10, 10), (5, 5), (3, 3)], 4, torch.float32, 0.3, ()),
    ('masked-fp16', 2, 9, 8, 32, 256, [(10, 15), (5, 8), (3, 4), (2, 2)], 4, torch.float16, 0.5, ()),
    ('masked-bf16-one-image-padded', 2, 10, 4, 16, 64, [(8, 12), (4, 6)], 8, torch.bfloat16, 0.2, (1,)),
]


def masked_case(i, B, Q, H, D, C, levels, P, dtype, frac, whole):
    inputs = list(make(B, Q, H, D, C, levels, P, dtype=dtype, bias=False, seed=100 + i))
    g = torch.Generator().manual_seed(200 + i)
    mask = torch.rand(B, inputs[0].shape[1], generator=g) < frac
    for b in whole:
        mask[b] = True
    return inputs, mask


def to_numpy(t):
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--upstream', default=os.environ.get('TINYDEFORM_UPSTREAM', ''))
    ap.add_argument('--out', default=os.path.join(HERE, 'golden_vectors.npz'))
    args = ap.parse_args()
    if not args.upstream:
        sys.exit('give --upstream <path to the upstream checkout>')
    sys.path.insert(0, args.upstream)
    from marearts_tinydeform.reference import ma_deform_attn_reference as upstream_reference

    cases = [(name, make(B, Q, H, D, C, levels, P, dtype=dtype, spread=spread, bias=bias, seed=i), dtype)
             for i, (name, B, Q, H, D, C, levels, P, dtype, spread, bias) in enumerate(SMALL_CASES)]
    cases.append(('boundary-locations', boundary_case(), torch.float32))
    arrays, manifest = {}, []
    with torch.no_grad():
        for i, (name, B, Q, H, D, C, levels, P, dtype, frac, whole) in enumerate(MASKED_CASES):
            inputs, mask = masked_case(i, B, Q, H, D, C, levels, P, dtype, frac, whole)
            zeroed = list(upcast(inputs))
            zeroed[0] = zeroed[0].masked_fill(mask[..., None], 0)
            ref64 = upstream_reference(*zeroed)
            key = name
            for field, t in zip(NAMES, inputs):
                if t is not None:
                    arrays[f'{key}/{field}'] = to_numpy(t)
            arrays[f'{key}/value_padding_mask'] = mask.numpy().astype(np.uint8)
            arrays[f'{key}/expected_f64'] = ref64.numpy()
            manifest.append({'key': key, 'dtype': str(dtype).replace('torch.', ''), 'bias': False,
                             'shape': list(ref64.shape), 'masked': True})
        for name, inputs, dtype in cases:
            ref64 = upstream_reference(*upcast(inputs))
            key = name.replace(' ', '_')
            for field, t in zip(NAMES, inputs):
                if t is not None:
                    arrays[f'{key}/{field}'] = to_numpy(t)
            arrays[f'{key}/expected_f64'] = ref64.numpy()
            if dtype == torch.float32:
                arrays[f'{key}/expected_native'] = upstream_reference(*inputs).numpy()
            manifest.append({'key': key, 'dtype': str(dtype).replace('torch.', ''),
                             'bias': inputs[2] is not None, 'shape': list(ref64.shape)})
    arrays['manifest'] = np.frombuffer(json.dumps(manifest).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **arrays)
    print(f'wrote {len(manifest)} cases to {args.out} ({os.path.getsize(args.out)} bytes)')


if __name__ == '__main__':
    main()
