"""marearts-tinydeform on B200: value projection + multi-scale deformable attention for DETR-style decoders.

The operator of upstream ``marearts_tinydeform`` (``marearts_tinydeform/__init__.py:1-79``), computed by hand-written
sm_100a kernels behind a C ABI (include/tinydeform.h). The drop-in for upstream's callers is the import name
``marearts_tinydeform``, whose ``ma_deform_attn`` keeps upstream's contract exactly (inference only); this package's
own ``ma_deform_attn`` takes the same arguments plus the additions below and also differentiates:

    ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                   sampling_locations, attention_weights, mode='auto')  -> [B, Q, H * D]

  mode='fused'    gather memory rows first, then project one vector per (query, head)
  mode='project'  project every memory token (our own GEMM kernel), then sample per head
  mode='auto'     choose_mode() picks one from the shapes, with crossovers measured on B200

Around the operator (additions; upstream has only the operator):

    deform_attn_layer(query, reference_points, memory, spatial_shapes, level_start_index, n_heads, n_points,
                      sampling_weight, sampling_bias, value_weight, value_bias, ...)   -> [B, Q, H * D | C_out]
    sampling_producer(query, reference_points, spatial_shapes, n_heads, n_points, sampling_weight, sampling_bias)
        -> sampling_locations, attention_weights
    pack_sampling_weights(offset_weight, offset_bias, attention_weight, attention_bias) -> the packed pair

the whole MSDeformAttn layer (query -> offsets and softmaxed weights -> attention -> output_proj) in one library call.

CPU tensors run ``ma_deform_attn_reference`` (as upstream does). CUDA tensors run only the native library; if it is
missing, the call raises. Unlike upstream (inference only), this package's ``ma_deform_attn`` differentiates CUDA
inputs that require grad: the forward runs the same kernels and the backward runs this library's backward kernels
(``autograd.py``).
"""

import functools

import torch

from . import _native
from .autograd import linear_train, ma_deform_attn_train, producer_train
from .reference import deform_attn_layer_reference, ma_deform_attn_reference, sampling_producer_reference

__all__ = ['ma_deform_attn', 'ma_deform_attn_reference', 'choose_mode', 'deform_attn_layer', 'sampling_producer',
           'pack_sampling_weights', 'deform_attn_layer_reference', 'sampling_producer_reference']
__version__ = '0.1.1+b200'

MODES = ('auto', 'fused', 'project')

# auto picks 'fused' while   queries * levels * points * 4 / (tokens * head_dim)  <  a + b / batch
# (upstream marearts_tinydeform/__init__.py:22-30, 39-46). 'fused' costs ~ batch * queries * samples * C row reads,
# 'project' ~ batch * tokens * C * H * D plus a fixed part that matters at batch 1.
# FUSED_LIMIT and FUSED_LIMIT_SM75 are upstream's tables (RTX 4090 / RTX 2080 Super); FUSED_LIMIT_SM100 is fitted
# to crossovers measured with this library on B200 (bench.py --sweep over upstream's query/batch grid, c4 and the
# c5 grid, 114 cases; profiles/auto_sweep_b200.md), used for compute capability 10.x. float32: the pick is within
# 10 % of the faster order in all 38 cases -- the fused order (a warp per row) wins up to about 300 queries per image
# at every batch, as the float32 projection runs three TF32 products per K step. float16 / bfloat16: 74 of 76; the
# fused order wins at 50-100 queries at batch 1-8 (RT-DETR shapes) and at batch 64 with 50 queries (c5), the project
# order above; no (a, b) also takes DINO batch 1 with 300 queries (fused 10.7 against 13.5 us), since the c5 shapes
# at batch 4-8 need the limit below its ratio.
FUSED_LIMIT = {torch.float32: (0.073, 0.032), torch.float16: (0.023, 0.031), torch.bfloat16: (0.023, 0.031)}
FUSED_LIMIT_SM75 = {torch.float32: (0.068, 0.0), torch.float16: (0.020, 0.0), torch.bfloat16: (0.132, 0.0)}
FUSED_LIMIT_SM100 = {torch.float32: (0.0775, 0.028), torch.float16: (0.024, -0.006), torch.bfloat16: (0.024, -0.006)}


@functools.lru_cache(maxsize=None)
def _limits(device_index):
    major, _ = torch.cuda.get_device_capability(device_index)
    if major == 10:
        return FUSED_LIMIT_SM100
    return FUSED_LIMIT if major >= 8 else FUSED_LIMIT_SM75


def choose_mode(memory, value_weight, sampling_locations):
    """The mode 'auto' runs: 'fused' for few queries per image, 'project' (project every token first) for many."""
    _, n_qry, n_head, n_lvl, n_pt, _ = sampling_locations.shape
    return _pick(memory, value_weight, n_qry, n_head, n_lvl, n_pt)


def _pick(memory, value_weight, n_qry, n_head, n_lvl, n_pt, limits=None):
    n_img, n_tok, _ = memory.shape
    head_dim = value_weight.shape[0] // n_head
    if limits is None:
        limits = _limits(memory.get_device()) if memory.is_cuda else FUSED_LIMIT
    a, b = limits.get(memory.dtype, limits[torch.float16])
    ratio = n_qry * n_lvl * n_pt * 4 / max(n_tok * head_dim, 1)
    return 'fused' if ratio < a + b / max(n_img, 1) else 'project'


def _outproj_in_epilogue(memory, value_weight, n_qry, n_head, output_weight):
    """Whether the project order would run output_proj in the sampler's cluster epilogue (td_set_output_proj_plan's
    automatic plan; the conditions of sample_outproj_kernel's 16-bit form)."""
    if output_weight is None or not memory.is_cuda or memory.dtype not in (torch.float16, torch.bfloat16):
        return False
    if _native.output_proj_plan() == _native.OUTPROJ_CHAINED:
        return False
    e = memory.element_size()
    hd = value_weight.shape[0]
    row = hd // n_head * e
    if hd * e != 512 or 8 % n_head or output_weight.shape[0] > 256:
        return False
    if row % 16 or row > 512 or (row // 16) & (row // 16 - 1):
        return False
    sms = torch.cuda.get_device_properties(memory.device).multi_processor_count
    return -(-memory.shape[0] * n_qry * n_head // 8) <= 3 * sms


def _pick_with_outproj(memory, value_weight, n_qry, n_head, n_lvl, n_pt, output_weight):
    """auto with output_proj: at batch 1, when the project order would fold output_proj into the sampler's
    epilogue, the project order (measured on B200, float16, C_out = 256: 1 x 20 queries 8.2 against 8.9 us fused
    + chained GEMM, 1 x 50 8.4 / 9.1, 1 x 100 8.7 / 9.5; at batch 2 and more the fused order with the chained GEMM
    is faster, 2 x 100 11.1 / 12.7); otherwise the operator's own pick."""
    if memory.shape[0] == 1 and _outproj_in_epilogue(memory, value_weight, n_qry, n_head, output_weight):
        return 'project'
    return _pick(memory, value_weight, n_qry, n_head, n_lvl, n_pt)


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
    attention kernel (in the same library call in the project order), overlapping its start with it.
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
    if mode == 'auto':
        _, n_qry, n_head, n_lvl, n_pt, _ = sampling_locations.shape
        mode = _pick_with_outproj(memory, value_weight, n_qry, n_head, n_lvl, n_pt, output_weight)
    if _wants_grad(memory, value_weight, value_bias, sampling_locations, attention_weights, output_weight,
                   output_bias):
        # training: the same forward kernels behind autograd Functions whose backward runs this library's
        # backward kernels (autograd.py), output_proj included
        _native.check_geometry(memory, spatial_shapes, level_start_index, sampling_locations, attention_weights)
        _native.check_projection(memory, value_weight, value_bias, sampling_locations.shape[2])
        out = ma_deform_attn_train(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                   sampling_locations, attention_weights, mode, value_padding_mask)
        if output_weight is None:
            return out
        _native.check_output_proj(output_weight, output_bias, out.shape[-1], out)
        return linear_train(out, output_weight, output_bias)
    if mode == 'project':
        # output_proj, if any, in the same library call
        return _native.project_forward(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                       sampling_locations, attention_weights, value_padding_mask, output_weight,
                                       output_bias)
    out = _native.fused_forward(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                sampling_locations, attention_weights, value_padding_mask)
    return out if output_weight is None else _native.linear(out, output_weight, output_bias)


def _wants_grad(*ts):
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts)


def pack_sampling_weights(offset_weight, offset_bias, attention_weight, attention_bias):
    """The layer's two query projections as one: sampling_offsets ([2 * H * L * P, Cq], rows (head, level, point,
    x/y)) stacked over attention_weights ([H * L * P, Cq], rows (head, level, point)), as the nn.Linear modules of
    Deformable-DETR's MSDeformAttn hold them. Pack once per model, not per call."""
    weight = torch.cat([offset_weight, attention_weight], 0)
    bias = None
    if offset_bias is not None or attention_bias is not None:
        zeros = offset_weight.new_zeros
        bias = torch.cat([offset_bias if offset_bias is not None else zeros(offset_weight.shape[0]),
                          attention_bias if attention_bias is not None else zeros(attention_weight.shape[0])])
    return weight, bias


def sampling_producer(query, reference_points, spatial_shapes, n_heads, n_points, sampling_weight, sampling_bias):
    """sampling_locations [B, Q, H, L, P, 2] and attention_weights [B, Q, H, L, P] from the query [B, Q, Cq] and
    reference points [B, Q, L, 2] (x, y) or reference boxes [B, Q, L, 4] (cx, cy, w, h), as
    sampling_producer_reference defines them. CUDA: the projection kernel, then the producer kernel."""
    if not query.is_cuda:
        return sampling_producer_reference(query, reference_points, spatial_shapes, n_heads, n_points,
                                           sampling_weight, sampling_bias)
    _native.load()
    L = spatial_shapes.shape[0]
    if sampling_weight.dim() != 2 or sampling_weight.shape[0] != 3 * n_heads * L * n_points:
        raise RuntimeError('sampling_weight must be [3 * H * L * P, Cq]: the offset rows, then the attention rows')
    if _wants_grad(query, reference_points, sampling_weight, sampling_bias):
        # training: the same kernels behind autograd Functions whose backward runs this library's kernels (the
        # producer's backward, then the query projection's gradient GEMMs)
        return producer_train(query, reference_points, spatial_shapes, n_heads, n_points, sampling_weight,
                              sampling_bias)
    proj = _native.linear(query, sampling_weight, sampling_bias)
    return _native.sampling_producer(proj, reference_points, spatial_shapes, n_heads, n_points)


def deform_attn_layer(query, reference_points, memory, spatial_shapes, level_start_index, n_heads, n_points,
                      sampling_weight, sampling_bias, value_weight, value_bias, output_weight=None, output_bias=None,
                      value_padding_mask=None, mode='auto'):
    """One multi-scale deformable attention layer (the forward of Deformable-DETR's MSDeformAttn, whose core is
    ma_deform_attn): [B, Q, H * D], or [B, Q, C_out] with output_weight.

    query [B, Q, Cq]; reference_points [B, Q, L, 2] or [B, Q, L, 4]; memory [B, N, C] (the value input);
    sampling_weight / sampling_bias: pack_sampling_weights of the offset and attention-weight projections;
    value_weight / value_bias: value_proj; output_weight / output_bias: output_proj (optional);
    value_padding_mask: bool [B, N], True = padded token. Same result as deform_attn_layer_reference.

    CUDA, mode 'project' (or 'auto' choosing it): three kernels in one library call (query projection, value
    projection, and the sampler computing the softmax and locations in its prologue), plus the output projection.
    Mode 'fused': query projection, producer kernel, fused gather-then-project kernel.
    """
    if mode not in MODES:
        raise ValueError(f'mode must be one of {MODES}, got {mode!r}')
    if output_bias is not None and output_weight is None:
        raise ValueError('output_bias needs output_weight')
    if not memory.is_cuda:
        return deform_attn_layer_reference(query, reference_points, memory, spatial_shapes, level_start_index,
                                           n_heads, n_points, sampling_weight, sampling_bias, value_weight,
                                           value_bias, output_weight, output_bias, value_padding_mask)
    _native.load()
    if mode == 'auto':
        mode = _pick_with_outproj(memory, value_weight, query.shape[1], n_heads, spatial_shapes.shape[0], n_points,
                                  output_weight)
    if _wants_grad(query, reference_points, memory, sampling_weight, sampling_bias, value_weight, value_bias,
                   output_weight, output_bias):
        # training: the producer and the attention behind autograd Functions on this library's kernels
        loc, attn = sampling_producer(query, reference_points, spatial_shapes, n_heads, n_points, sampling_weight,
                                      sampling_bias)
        return ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index, loc, attn,
                              mode=mode, value_padding_mask=value_padding_mask, output_weight=output_weight,
                              output_bias=output_bias)
    return _native.layer_forward(query, reference_points, memory, spatial_shapes, level_start_index, n_heads,
                                 n_points, sampling_weight, sampling_bias, value_weight, value_bias, output_weight,
                                 output_bias, value_padding_mask, order=mode)
