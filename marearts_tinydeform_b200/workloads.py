"""The benchmark workloads: decoder-layer shapes and seeded synthetic inputs for ma_deform_attn.

There is no dataset behind these numbers: RT-DETR / DINO decoder layers are plain tensor shapes, and the inputs are
seeded synthetic tensors with the distributions below (one torch.Generator per call, on CPU, then moved).

  c1   RT-DETR 640x640, float32, B=1, Q=300, C=256, H=8, D=32, L=3 (80x80, 40x40, 20x20; N=8400), P=4
  c1h  the same shapes in float16 (the B=1, Q=300 fp16 north-star call)
  c2   RT-DETR shapes, float16, B=1, Q=100, locations U(-0.05, 1.05), value_bias None on odd seeds
  c3   RT-DETR shapes, bfloat16, B=8, Q=300
  c4   DINO 800x1333, float16, B=8, Q=900, L=4 (100x167, 50x84, 25x42, 13x21; N=22223), P=4
  c5   stress: L=4 (80x80 .. 10x10; N=8500), P=16, C=512, H=8, D=64, B in {1,4,8,64}, Q in {50,100,300,900}

memory ~ N(0, 1) (c5: variance 2, i.e. std sqrt(2)); value_weight xavier-uniform (c5: N(0, 1/C), i.e. std
1/sqrt(C)); value_bias ~ U(-0.05, 0.05); sampling_locations ~ U(0, 1) unless stated; attention_weights = softmax over
the L*P entries of N(0, 1) logits.
"""

import math

import torch

RTDETR_LEVELS = [(80, 80), (40, 40), (20, 20)]
DINO_LEVELS = [(100, 167), (50, 84), (25, 42), (13, 21)]
STRESS_LEVELS = [(80, 80), (40, 40), (20, 20), (10, 10)]

CONFIGS = {
    'c1': dict(B=1, Q=300, C=256, H=8, D=32, levels=RTDETR_LEVELS, P=4, dtype=torch.float32),
    'c1h': dict(B=1, Q=300, C=256, H=8, D=32, levels=RTDETR_LEVELS, P=4, dtype=torch.float16),
    'c2': dict(B=1, Q=100, C=256, H=8, D=32, levels=RTDETR_LEVELS, P=4, dtype=torch.float16,
               loc_range=(-0.05, 1.05), bias_on_odd_seeds=False),
    'c3': dict(B=8, Q=300, C=256, H=8, D=32, levels=RTDETR_LEVELS, P=4, dtype=torch.bfloat16),
    'c4': dict(B=8, Q=900, C=256, H=8, D=32, levels=DINO_LEVELS, P=4, dtype=torch.float16),
    'c5': dict(B=8, Q=300, C=512, H=8, D=64, levels=STRESS_LEVELS, P=16, dtype=torch.float16,
               loc_range=(-0.1, 1.1), memory_std=math.sqrt(2.0), weight='normal'),
}
C5_BATCHES = (1, 4, 8, 64)
C5_QUERIES = (50, 100, 300, 900)


def level_tensors(levels, device='cpu'):
    shapes = torch.tensor(levels, dtype=torch.long)
    starts = torch.zeros(len(levels), dtype=torch.long)
    if len(levels) > 1:
        starts[1:] = (shapes[:, 0] * shapes[:, 1]).cumsum(0)[:-1]
    return shapes.to(device), starts.to(device)


def n_tokens(levels):
    return sum(h * w for h, w in levels)


def make_inputs(name, seed=0, device='cpu', generate_on_device=False, **overrides):
    """Seeded inputs of config `name` (keys of CONFIGS), with any field overridden (B, Q, dtype, ...).

    Returns (memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
    attention_weights) on `device`. By default the numbers come from a CPU generator (identical on every machine);
    generate_on_device=True draws them with a generator on `device` instead (fast, for timing only).
    """
    cfg = dict(CONFIGS[name])
    cfg.update(overrides)
    B, Q, C, H, D, P = cfg['B'], cfg['Q'], cfg['C'], cfg['H'], cfg['D'], cfg['P']
    levels, dtype = cfg['levels'], cfg['dtype']
    L, N, HD = len(levels), n_tokens(levels), H * D
    gdev = torch.device(device) if generate_on_device else torch.device('cpu')
    g = torch.Generator(device=gdev).manual_seed(seed)
    kw = dict(generator=g, device=gdev)
    memory = torch.randn(B, N, C, **kw) * cfg.get('memory_std', 1.0)
    if cfg.get('weight', 'xavier') == 'normal':
        weight = torch.randn(HD, C, **kw) / math.sqrt(C)
    else:
        bound = math.sqrt(6.0 / (HD + C))
        weight = (torch.rand(HD, C, **kw) * 2 - 1) * bound
    bias = (torch.rand(HD, **kw) * 2 - 1) * 0.05
    if 'bias_on_odd_seeds' in cfg and seed % 2 == 1:
        bias = None
    lo, hi = cfg.get('loc_range', (0.0, 1.0))
    loc = torch.rand(B, Q, H, L, P, 2, **kw) * (hi - lo) + lo
    attn = torch.randn(B, Q, H, L * P, **kw).softmax(-1).view(B, Q, H, L, P)
    shapes, starts = level_tensors(levels)
    out = [memory.to(dtype), weight.to(dtype), None if bias is None else bias.to(dtype), shapes, starts,
           loc.to(dtype), attn.to(dtype)]
    return [None if t is None else t.to(device) for t in out]


def algorithmic_bytes(B, Q, N, C, H, D, L, P, elem_bytes, bias=True):
    """Compulsory HBM bytes of one call, whatever the order: memory and W read once, loc + attn read, out written."""
    HD = H * D
    return elem_bytes * (B * N * C + HD * C + (HD if bias else 0) + 3 * B * Q * H * L * P + B * Q * HD)
