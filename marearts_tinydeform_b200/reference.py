"""The plain-PyTorch definition of the operator: project every memory token, then bilinear-sample per level.

This is the public ``ma_deform_attn_reference`` of the drop-in API (upstream
``marearts_tinydeform/reference.py:13-40``). It defines what ``ma_deform_attn`` returns: ``nn.Linear`` on every
memory token, then ``F.grid_sample`` with bilinear interpolation, zero padding and ``align_corners=False`` on each
level, then the attention-weighted sum over levels x points. It runs on CPU and GPU in any float dtype and supports
autograd (the CUDA path has its own backward kernel).

CPU tensors passed to ``ma_deform_attn`` come here, exactly as upstream ``marearts_tinydeform/__init__.py:62-64``
routes them. CUDA tensors never do: the CUDA path raises when its native library is missing.
"""

import torch
import torch.nn.functional as F


def ma_deform_attn_reference(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                             sampling_locations, attention_weights, value_padding_mask=None):
    """value = memory @ value_weight.T + value_bias, then multi-scale deformable attention.

    memory              [B, N, C]
    value_weight        [H * D, C]      (an nn.Linear weight)
    value_bias          [H * D] or None
    spatial_shapes      [L, 2] int64    (height, width) of each level; tokens are laid out level after level
    level_start_index   [L] int64       first token of each level
    sampling_locations  [B, Q, H, L, P, 2]  (x, y) normalised to [0, 1]
    attention_weights   [B, Q, H, L, P]     already normalised (softmax over L * P)
    value_padding_mask  [B, N] bool or None: True zeroes that token's projected value (Deformable-DETR's
                        input_padding_mask; an addition to the upstream signature, which has no mask)
    returns             [B, Q, H * D]
    """
    n_img, n_tok, _ = memory.shape
    _, n_qry, n_head, n_lvl, n_pt, _ = sampling_locations.shape
    value = F.linear(memory, value_weight, value_bias)                 # [B, N, H*D]
    if value_padding_mask is not None:
        value = value.masked_fill(value_padding_mask.to(torch.bool)[..., None], 0)
    head_dim = value.shape[-1] // n_head
    # grid_sample wants (x, y) in [-1, 1]; one image per (batch, head) pair, D channels each
    grid = sampling_locations.mul(2).sub(1).permute(0, 2, 1, 3, 4, 5)  # [B, H, Q, L, P, 2]
    grid = grid.reshape(n_img * n_head, n_qry, n_lvl, n_pt, 2)
    per_head = value.view(n_img, n_tok, n_head, head_dim).permute(0, 2, 3, 1)  # [B, H, D, N]
    per_head = per_head.reshape(n_img * n_head, head_dim, n_tok)
    sampled = []
    for lvl in range(n_lvl):
        # level geometry is read on the host, like any grid_sample caller
        height, width = int(spatial_shapes[lvl, 0]), int(spatial_shapes[lvl, 1])
        first = int(level_start_index[lvl])
        image = per_head[:, :, first:first + height * width].reshape(n_img * n_head, head_dim, height, width)
        sampled.append(F.grid_sample(image, grid[:, :, lvl], mode='bilinear', padding_mode='zeros',
                                     align_corners=False))             # [B*H, D, Q, P]
    stacked = torch.cat(sampled, dim=-1)                               # [B*H, D, Q, L*P]
    weights = attention_weights.permute(0, 2, 1, 3, 4).reshape(n_img * n_head, 1, n_qry, n_lvl * n_pt)
    out = (stacked * weights).sum(-1)                                  # [B*H, D, Q]
    return out.view(n_img, n_head * head_dim, n_qry).transpose(1, 2).contiguous()


def sampling_producer_reference(query, reference_points, spatial_shapes, n_heads, n_points, sampling_weight,
                                sampling_bias):
    """sampling_locations [B, Q, H, L, P, 2] and attention_weights [B, Q, H, L, P] of the multi-scale deformable
    attention layer (Deformable-DETR's MSDeformAttn, RT-DETR's decoder). sampling_weight = [W_offsets; W_attention]
    ([3 * H * L * P, Cq]; the offset rows ordered (head, level, point, x/y), the attention rows (head, level, point)),
    sampling_bias likewise. The logits are normalised by a softmax over the L * P points of each head, and the
    offsets move the reference points: ref + offset / (w_l, h_l) for reference_points [B, Q, L, 2],
    ref.xy + offset / P * ref.wh * 0.5 for reference boxes [B, Q, L, 4]. The upstream operator takes both results as
    inputs and has no producer."""
    B, Q, _ = query.shape
    L = spatial_shapes.shape[0]
    H, P = n_heads, n_points
    proj = F.linear(query, sampling_weight, sampling_bias)
    offsets = proj[..., :2 * H * L * P].reshape(B, Q, H, L, P, 2)
    logits = proj[..., 2 * H * L * P:].reshape(B, Q, H, L * P)
    attention = logits.softmax(-1).view(B, Q, H, L, P)
    if reference_points.shape[-1] == 2:
        norm = torch.stack([spatial_shapes[:, 1], spatial_shapes[:, 0]], -1).to(query.dtype)   # (w, h) per level
        loc = reference_points[:, :, None, :, None, :] + offsets / norm[None, None, None, :, None, :]
    else:
        loc = (reference_points[:, :, None, :, None, :2]
               + offsets / P * reference_points[:, :, None, :, None, 2:] * 0.5)
    return loc, attention


def deform_attn_layer_reference(query, reference_points, memory, spatial_shapes, level_start_index, n_heads,
                                n_points, sampling_weight, sampling_bias, value_weight, value_bias,
                                output_weight=None, output_bias=None, value_padding_mask=None):
    """One deformable attention layer with torch operators: the producer above, ma_deform_attn_reference, and the
    optional output projection."""
    loc, attention = sampling_producer_reference(query, reference_points, spatial_shapes, n_heads, n_points,
                                                 sampling_weight, sampling_bias)
    out = ma_deform_attn_reference(memory, value_weight, value_bias, spatial_shapes, level_start_index, loc,
                                   attention, value_padding_mask)
    return out if output_weight is None else F.linear(out, output_weight, output_bias)
