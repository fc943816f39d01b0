"""Shape cases and the seeded input generator of the parity tests.

The generator follows the input recipe of upstream's tests (tests/test_correctness.py:13-26): memory ~ N(0, 1),
value_weight ~ N(0, 1) / sqrt(C), value_bias ~ 0.1 * N(0, 1) (or None), each query gets a centre ~ U(0, 1)^2 and every
(head, level, point) location adds spread * 0.3 * N(0, 1) to it, which deliberately lands corners outside the map;
attention_weights are a softmax over L * P.
"""

import torch

# name, B, Q, H, D, C, levels, P -- the geometries upstream's tests cover (tests/test_correctness.py:33-43)
CASES = [
    ('rtdetr-640', 1, 300, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4),
    ('rtdetr-640 b4 few queries', 4, 40, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4),
    ('deformable-detr 4 levels non-square', 2, 100, 8, 32, 256, [(100, 152), (50, 76), (25, 38), (13, 19)], 4),
    ('narrow heads', 2, 50, 4, 16, 64, [(32, 48), (16, 24)], 8),
    ('one level many points', 1, 64, 2, 64, 128, [(20, 30)], 16),
    ('wide channels', 1, 40, 12, 64, 768, [(40, 40), (20, 20), (10, 10)], 4),
    ('odd channels', 2, 33, 3, 10, 30, [(13, 17), (7, 9)], 4),
    ('channels % 8 != 0, % 4 == 0', 1, 25, 4, 9, 36, [(11, 12)], 4),
]

# small cases with every kind of geometry, for the golden vectors and fast CPU checks
SMALL_CASES = [
    # name, B, Q, H, D, C, levels, P, dtype, spread, bias
    ('tiny', 1, 10, 2, 8, 16, [(6, 7), (3, 4)], 2, torch.float32, 1.0, True),
    ('rtdetr-mini', 1, 24, 8, 32, 256, [(10, 10), (5, 5), (3, 3)], 4, torch.float32, 1.0, True),
    ('four-levels-nonsquare-fp16', 2, 12, 8, 32, 256, [(10, 15), (5, 8), (3, 4), (2, 2)], 4, torch.float16, 1.0,
     True),
    ('narrow-heads-bf16', 2, 10, 4, 16, 64, [(8, 12), (4, 6)], 8, torch.bfloat16, 1.0, True),
    ('one-level-many-points', 1, 8, 2, 64, 128, [(5, 6)], 16, torch.float32, 1.0, True),
    ('wide-channels-fp16', 1, 4, 6, 64, 384, [(4, 4), (2, 2)], 4, torch.float16, 1.0, True),
    ('odd-channels', 2, 7, 3, 10, 30, [(5, 7), (3, 4)], 4, torch.float32, 1.0, True),
    ('channels-mod8-fp16', 1, 5, 4, 9, 36, [(4, 5)], 4, torch.float16, 1.0, True),
    ('far-outside', 2, 6, 4, 8, 32, [(5, 6), (3, 3)], 4, torch.float32, 200.0, True),
    ('no-bias', 1, 12, 8, 32, 256, [(6, 6), (3, 3)], 4, torch.float32, 1.0, False),
    ('max-level-points', 1, 4, 2, 16, 32, [(6, 6), (3, 3), (2, 2), (1, 1)], 16, torch.float32, 1.0, True),
    ('float64', 1, 9, 2, 8, 16, [(5, 4), (2, 3)], 3, torch.float64, 1.0, True),
]


def make(B, Q, H, D, C, levels, P, dtype=torch.float32, spread=1.0, bias=True, seed=0):
    """Seeded inputs (memory, value_weight, value_bias, spatial_shapes, level_start_index, loc, attn) on CPU."""
    g = torch.Generator().manual_seed(seed)
    shapes = torch.tensor(levels, dtype=torch.long)
    starts = torch.zeros(len(levels), dtype=torch.long)
    starts[1:] = (shapes[:, 0] * shapes[:, 1]).cumsum(0)[:-1]
    N = int((shapes[:, 0] * shapes[:, 1]).sum())
    L = len(levels)
    memory = torch.randn(B, N, C, generator=g)
    weight = torch.randn(H * D, C, generator=g) / C ** 0.5
    b = torch.randn(H * D, generator=g) * 0.1 if bias else None
    centre = torch.rand(B, Q, 1, 1, 1, 2, generator=g)
    loc = centre + spread * 0.3 * torch.randn(B, Q, H, L, P, 2, generator=g)
    attn = torch.randn(B, Q, H, L * P, generator=g).softmax(-1).view(B, Q, H, L, P)
    return [t if t is None or t.dtype == torch.long else t.to(dtype)
            for t in (memory, weight, b, shapes, starts, loc, attn)]


def boundary_case(dtype=torch.float32):
    """Locations exactly on pixel centres, pixel edges, the map border and just outside it (one level 4 x 5)."""
    g = torch.Generator().manual_seed(7)
    levels = [(4, 5), (2, 3)]
    shapes = torch.tensor(levels, dtype=torch.long)
    starts = torch.tensor([0, 20], dtype=torch.long)
    N, C, H, D, P = 26, 16, 2, 8, 4
    memory = torch.randn(1, N, C, generator=g)
    weight = torch.randn(H * D, C, generator=g) / C ** 0.5
    b = torch.randn(H * D, generator=g) * 0.1
    xs = [0.0, 1.0, 0.1, 0.5, 0.3, 0.7, 1.0 / 3, 0.999999, 1e-7, -0.1, 1.1, 0.9]
    ys = [0.0, 1.0, 0.25, 0.5, 0.125, 0.875, 0.6, 0.0, 1.0, 1.05, -0.05, 0.75]
    Q = len(xs)
    loc = torch.zeros(1, Q, H, 2, P, 2)
    for q, (x, y) in enumerate(zip(xs, ys)):
        for p in range(P):
            loc[0, q, :, :, p, 0] = x if p % 2 == 0 else 1.0 - x
            loc[0, q, :, :, p, 1] = y if p < 2 else 1.0 - y
    attn = torch.randn(1, Q, H, 2 * P, generator=g).softmax(-1).view(1, Q, H, 2, P)
    return [t if t.dtype == torch.long else t.to(dtype) for t in (memory, weight, b, shapes, starts, loc, attn)]


def to(args, device):
    return [None if t is None else t.to(device) for t in args]


def upcast(args):
    """The float64 copy the oracle is run on for float16 / bfloat16 inputs (upstream tests/test_correctness.py:79)."""
    return [t if t is None or t.dtype == torch.long else t.double() for t in args]


# name, B, Q, Cq, H, D, C, levels, P -- decoder-layer geometries for the sampling producer and the whole layer
LAYER_CASES = [
    ('rtdetr-640 layer', 1, 300, 256, 8, 32, 256, [(80, 80), (40, 40), (20, 20)], 4),
    ('deformable-detr 4 levels b2', 2, 100, 256, 8, 32, 256, [(50, 76), (25, 38), (13, 19), (7, 10)], 4),
    ('narrow, query wider than memory', 2, 40, 128, 4, 16, 64, [(16, 24), (8, 12)], 8),
    ('max level points', 1, 20, 64, 2, 16, 32, [(12, 12), (6, 6), (3, 3), (2, 2)], 16),
    ('odd sizes', 2, 17, 40, 3, 10, 30, [(9, 11), (5, 6)], 3),
]


def make_layer(B, Q, Cq, H, D, C, levels, P, ref_dim=2, dtype=torch.float32, bias=True, seed=0):
    """Seeded inputs of one deformable attention layer on CPU: (query, reference_points, memory, spatial_shapes,
    level_start_index, sampling_weight, sampling_bias, value_weight, value_bias). Offsets come out ~ N(0, 2) pixels
    (2-d) or ~ N(0, 2 P) box-halves (4-d); logits ~ N(0, 1.5); reference points ~ U(0, 1), boxes' w, h ~ U(0.05, 0.5)."""
    g = torch.Generator().manual_seed(seed)
    shapes = torch.tensor(levels, dtype=torch.long)
    starts = torch.zeros(len(levels), dtype=torch.long)
    starts[1:] = (shapes[:, 0] * shapes[:, 1]).cumsum(0)[:-1]
    N = int((shapes[:, 0] * shapes[:, 1]).sum())
    L = len(levels)
    query = torch.randn(B, Q, Cq, generator=g)
    memory = torch.randn(B, N, C, generator=g)
    off_scale = 2.0 if ref_dim == 2 else 0.3 * P
    w_off = torch.randn(2 * H * L * P, Cq, generator=g) * (off_scale / Cq ** 0.5)
    w_att = torch.randn(H * L * P, Cq, generator=g) * (1.5 / Cq ** 0.5)
    sampling_weight = torch.cat([w_off, w_att])
    sampling_bias = torch.randn(3 * H * L * P, generator=g) * 0.5 if bias else None
    value_weight = torch.randn(H * D, C, generator=g) / C ** 0.5
    value_bias = torch.randn(H * D, generator=g) * 0.1 if bias else None
    if ref_dim == 2:
        ref = torch.rand(B, Q, L, 2, generator=g)
    else:
        ref = torch.cat([torch.rand(B, Q, L, 2, generator=g), 0.05 + 0.45 * torch.rand(B, Q, L, 2, generator=g)], -1)
    return [t if t is None or t.dtype == torch.long else t.to(dtype)
            for t in (query, ref, memory, shapes, starts, sampling_weight, sampling_bias, value_weight, value_bias)]
