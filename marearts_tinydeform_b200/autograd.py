"""Training support: ma_deform_attn (and output_proj) on CUDA tensors that require grad.

Upstream's CUDA operator is inference only (marearts_tinydeform/__init__.py:67-71 rejects inputs that require
grad); this build differentiates it, on this library's kernels only. Forward: the same B200 kernels as inference,
in the order `mode` picks, saving the inputs and, in the project order, the projected value the forward computed
anyway (head-major, B * N * H * D elements kept until the backward). Backward:

    value (fused order only)   td_value_proj: the value projection again, head-major
    grad_value, grad_loc,      td_sample_backward: one pass over every sampling point (float32 accumulation)
      grad_attn
    grad_value in the dtype,   td_grad_value_finish: one pass over the float32 accumulator
      grad_value_bias
    grad_memory                td_linear_grad_input:  grad_value @ value_weight          (tcgen05 for 16-bit types)
    grad_value_weight          td_linear_grad_weight: grad_value^T @ memory, over every token of every image

grad_value is rounded once from its float32 accumulator for float16 / bfloat16 inputs, as autograd's own
half-precision backward keeps its gradients in half precision; float32 / float64 inputs keep float32 / float64. The
value padding mask blocks the gradient of padded tokens exactly as masked_fill does in the reference.

LinearFunction is output_proj (y = x @ W^T + b) on the same kernels: td_linear forward, td_linear_grad_input and
td_linear_grad_weight (with the bias gradient's column sums) backward. It is also the query projection of the
sampling producer, whose own step (softmax over each row's L * P logits, offsets moving the reference points) is
ProducerFunction: td_sampling_producer forward, td_sampling_producer_backward backward (gradients of the query
projection's output and of the reference points).
"""

import torch

from . import _native


class MaDeformAttnFunction(torch.autograd.Function):
    """out = ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index,
    sampling_locations, attention_weights) on CUDA, differentiable in the five float inputs."""

    @staticmethod
    def forward(ctx, memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
                attention_weights, mode, value_padding_mask):
        value = None
        if mode == 'fused':
            out = _native.fused_forward(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                        sampling_locations, attention_weights, value_padding_mask)
        else:
            out, value = _native.project_forward(memory, value_weight, value_bias, spatial_shapes,
                                                 level_start_index, sampling_locations, attention_weights,
                                                 value_padding_mask, return_value=True)
        ctx.save_for_backward(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                              sampling_locations, attention_weights, value_padding_mask, value)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        memory, weight, bias, shapes, starts, loc, attn, mask, value_hm = ctx.saved_tensors
        need = ctx.needs_input_grad
        H = loc.shape[2]
        B, N, C = memory.shape
        HD = weight.shape[0]
        g = grad_out if grad_out.dtype == memory.dtype else grad_out.to(memory.dtype)
        if value_hm is None:  # the fused order never formed the value: project it again, head-major
            value_hm = _native.value_proj(memory, weight, bias, H, head_major=True)
        grad_value, grad_loc, grad_attn = _native.sample_backward(value_hm, shapes, starts, loc, attn, g, mask)
        acc = grad_value.view(B * N, HD)
        want_bias = bias is not None and need[2]
        # the rounding to the dtype and the bias gradient's column sums in one pass over the accumulator
        done = _native.grad_value_finish(acc, memory.dtype, want_bias) if memory.dtype != torch.float64 else None
        if done is not None:
            gv, bias_sum = done
        else:  # float64, or a width the finishing kernel does not take: the column sums come with grad_W
            gv = acc if acc.dtype == memory.dtype else acc.to(memory.dtype)
            bias_sum = None
        grad_memory = grad_weight = grad_bias = None
        if need[0]:
            grad_memory = _native.linear_grad_input(gv, weight).view(B, N, C)
        if need[1] or (want_bias and bias_sum is None):
            gw, gb = _native.linear_grad_weight(gv, memory.reshape(B * N, C), with_bias=want_bias and bias_sum is None)
            grad_weight = gw if need[1] else None
            if gb is not None:
                bias_sum = gb
        if want_bias:
            grad_bias = bias_sum if bias_sum.dtype == bias.dtype else bias_sum.to(bias.dtype)
        return (grad_memory, grad_weight, grad_bias, None, None, grad_loc if need[5] else None,
                grad_attn if need[6] else None, None, None)


def ma_deform_attn_train(memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
                         attention_weights, mode, value_padding_mask=None):
    """The differentiable CUDA call (mode 'fused' or 'project' for the forward)."""
    mask = _native.check_mask(value_padding_mask, memory)
    return MaDeformAttnFunction.apply(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                      sampling_locations, attention_weights, mode, mask)


class LinearFunction(torch.autograd.Function):
    """y = x @ weight.T + bias over the last dimension of x, forward and backward on this library's kernels."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        ctx.save_for_backward(x, weight, bias)
        return _native.linear(x, weight, bias)

    @staticmethod
    def backward(ctx, grad_y):
        x, weight, bias = ctx.saved_tensors
        need = ctx.needs_input_grad
        g = grad_y if grad_y.dtype == x.dtype else grad_y.to(x.dtype)
        grad_x = _native.linear_grad_input(g, weight) if need[0] else None
        grad_w = grad_b = None
        want_bias = bias is not None and need[2]
        if need[1] or want_bias:
            gw, gb = _native.linear_grad_weight(g, x, with_bias=want_bias)
            grad_w = gw if need[1] else None
            grad_b = gb
        return grad_x, grad_w, grad_b


def linear_train(x, weight, bias):
    """The differentiable output_proj on CUDA."""
    return LinearFunction.apply(x, weight, bias)


class ProducerFunction(torch.autograd.Function):
    """(sampling_locations, attention_weights) from the query projection proj [B, Q, 3 * H * L * P] and the reference
    points, on this library's producer kernels, differentiable in proj and the reference points."""

    @staticmethod
    def forward(ctx, proj, reference_points, spatial_shapes, heads, points):
        ctx.save_for_backward(proj, reference_points, spatial_shapes)
        ctx.heads, ctx.points = heads, points
        loc, attn = _native.sampling_producer(proj, reference_points, spatial_shapes, heads, points)
        return loc, attn

    @staticmethod
    def backward(ctx, grad_loc, grad_attn):
        proj, ref, shapes = ctx.saved_tensors
        need = ctx.needs_input_grad
        if not (need[0] or need[1]):
            return None, None, None, None, None
        grad_proj, grad_ref = _native.sampling_producer_backward(proj, ref, shapes, ctx.heads, ctx.points, grad_loc,
                                                                 grad_attn, want_ref=need[1])
        return grad_proj if need[0] else None, grad_ref, None, None, None


def producer_train(query, reference_points, spatial_shapes, heads, points, sampling_weight, sampling_bias):
    """The differentiable sampling producer on CUDA: the query projection (LinearFunction), then ProducerFunction."""
    proj = LinearFunction.apply(query, sampling_weight, sampling_bias)
    return ProducerFunction.apply(proj, reference_points, spatial_shapes, heads, points)
