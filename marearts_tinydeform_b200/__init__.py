"""marearts-tinydeform on B200: value projection + multi-scale deformable attention for DETR-style decoders.

A drop-in for upstream ``marearts_tinydeform`` (``marearts_tinydeform/__init__.py:1-79``): the same public names,
arguments, results and errors, computed by hand-written sm_100a kernels behind a C ABI (include/tinydeform.h):

    ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                   sampling_locations, attention_weights, mode='auto')  -> [B, Q, H * D]

  mode='fused'    gather memory rows first, then project one vector per (query, head)
  mode='project'  project every memory token (our own GEMM kernel), then sample per head
  mode='auto'     choose_mode() picks one from the shapes, with crossovers measured on B200

CPU tensors run ``ma_deform_attn_reference`` (as upstream does). CUDA tensors run only the native library; if it is
missing, the call raises. Inference only: inputs that require grad are rejected.
"""

import functools

import torch

from . import _native
from .reference import ma_deform_attn_reference

__all__ = ['ma_deform_attn', 'ma_deform_attn_reference', 'choose_mode']
__version__ = '0.1.1+b200'

MODES = ('auto', 'fused', 'project')

# auto picks 'fused' while   queries * levels * points * 4 / (tokens * head_dim)  <  a + b / batch
# (upstream marearts_tinydeform/__init__.py:22-30, 39-46). 'fused' costs ~ batch * queries * samples * C row reads,
# 'project' ~ batch * tokens * C * H * D plus a fixed part that matters at batch 1.
# FUSED_LIMIT and FUSED_LIMIT_SM75 are upstream's tables (RTX 4090 / RTX 2080 Super); FUSED_LIMIT_SM100 is fitted
# to crossovers measured with this library on B200 (bench.py --sweep over upstream's query/batch grid, c4 and the
# c5 grid: 114 cases, the pick within 10% of the faster order in all of them), used for compute capability 10.x.
# On B200 the tensor-core projection (float32 too, as three TF32 products) makes 'project' cheap even at batch 1,
# while 'fused' pays its per-call latency once for the whole batch, so 'fused' only wins at batch >= 4 with few
# queries: b is negative (the limit grows with the batch).
FUSED_LIMIT = {torch.float32: (0.073, 0.032), torch.float16: (0.023, 0.031), torch.bfloat16: (0.023, 0.031)}
FUSED_LIMIT_SM75 = {torch.float32: (0.068, 0.0), torch.float16: (0.020, 0.0), torch.bfloat16: (0.132, 0.0)}
FUSED_LIMIT_SM100 = {torch.float32: (0.026, -0.05), torch.float16: (0.015, -0.024), torch.bfloat16: (0.015, -0.024)}


@functools.lru_cache(maxsize=None)
def _limits(device_index):
    major, _ = torch.cuda.get_device_capability(device_index)
    if major == 10:
        return FUSED_LIMIT_SM100
    return FUSED_LIMIT if major >= 8 else FUSED_LIMIT_SM75


def choose_mode(memory, value_weight, sampling_locations):
    """The mode 'auto' runs: 'fused' for few queries per image, 'project' (project every token first) for many."""
    n_img, n_tok, _ = memory.shape
    _, n_qry, n_head, n_lvl, n_pt, _ = sampling_locations.shape
    head_dim = value_weight.shape[0] // n_head
    limits = _limits(memory.get_device()) if memory.is_cuda else FUSED_LIMIT
    a, b = limits.get(memory.dtype, limits[torch.float16])
    ratio = n_qry * n_lvl * n_pt * 4 / max(n_tok * head_dim, 1)
    return 'fused' if ratio < a + b / max(n_img, 1) else 'project'


def ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                   sampling_locations, attention_weights, mode='auto', value_padding_mask=None,
                   output_weight=None, output_bias=None):
    """value = memory @ value_weight.T + value_bias, then multi-scale deformable attention; [B, Q, H * D].

    Same arguments, shapes and result as ma_deform_attn_reference (grid_sample, bilinear, zero padding,
    align_corners=False). CUDA tensors (float32, float16, bfloat16, float64; float32 accumulation, float64 for
    float64) run the B200 kernels in the order `mode` names; CPU tensors run the reference.

    value_padding_mask (an addition; the upstream operator has none): bool [B, N], True = padded token. As
    Deformable-DETR's input_padding_mask, the projected value of a padded token is zeroed (its bias included)
    before sampling, so it contributes nothing.

    output_weight / output_bias (an addition): the decoder's output_proj (an nn.Linear [C_out, H * D]) applied to the
    result, so the call returns [B, Q, C_out]; on CUDA it runs as a tensor-core GEMM queued right behind the
    attention kernel, overlapping its start with it.
    """
    if mode not in MODES:
        raise ValueError(f'mode must be one of {MODES}, got {mode!r}')
    if output_bias is not None and output_weight is None:
        raise ValueError('output_bias needs output_weight')
    if not memory.is_cuda:
        out = ma_deform_attn_reference(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                       sampling_locations, attention_weights, value_padding_mask)
        return out if output_weight is None else torch.nn.functional.linear(out, output_weight, output_bias)
    _native.load()  # raises RuntimeError when the native library is missing: there is no fallback
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad
            for t in (memory, value_weight, value_bias, sampling_locations, attention_weights, output_weight,
                      output_bias)):
        raise RuntimeError('ma_deform_attn is inference only: run it under torch.no_grad() / '
                           'torch.inference_mode(), or use ma_deform_attn_reference for training')
    if mode == 'auto':
        mode = choose_mode(memory, value_weight, sampling_locations)
    run = _native.fused_forward if mode == 'fused' else _native.project_forward
    out = run(memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
              attention_weights, value_padding_mask)
    return out if output_weight is None else _native.linear(out, output_weight, output_bias)
