"""Training support: ma_deform_attn on CUDA tensors that require grad.

Upstream's CUDA operator is inference only (marearts_tinydeform/__init__.py:67-71 rejects inputs that require
grad); this build differentiates it. Forward: the same B200 kernels as inference, in the order `mode` picks,
saving the inputs and, in the project order, the projected value the forward computed anyway (head-major, B * N *
H * D elements kept until the backward). Backward: in the fused order the value projection is run again
(nn.Linear layout, by torch's GEMM: the backward runs on autograd's worker thread, also under CUDA-graph capture,
where a library GEMM needs no tensor-map set-up); then td_sample_backward gives grad_value (float32 accumulation),
grad_sampling_locations and grad_attention_weights in one pass, and the three parameter gradients follow by plain
GEMMs and a column sum:

    grad_memory       = grad_value @ value_weight
    grad_value_weight = grad_value^T @ memory          (summed over every token of every image)
    grad_value_bias   = sum of grad_value over tokens

These two GEMMs are library GEMMs (torch.matmul, cuBLAS) in the inputs' dtype -- grad_value is rounded once from
its float32 accumulator, as autograd's own half-precision backward keeps its gradients in half precision, and the
tensor cores then run them -- except for float32 / float64 inputs, which keep float32 / float64; the bias gradient
is summed from the float32 accumulator, in the same pass as that rounding (td_grad_value_finish). The value
padding mask blocks the gradient of padded tokens exactly as masked_fill does in the reference.
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
        g = grad_out.to(memory.dtype).contiguous()
        if value_hm is not None:  # the forward's own value, head-major
            grad_value, grad_loc, grad_attn = _native.sample_backward(value_hm, shapes, starts, loc, attn, g, mask)
        else:  # the fused order never formed the value: project it again, head-major, with the library's GEMM
            value = _native.value_proj(memory, weight, bias, H, head_major=True)
            grad_value, grad_loc, grad_attn = _native.sample_backward(value, shapes, starts, loc, attn, g, mask)
        acc = grad_value.view(B * N, HD)
        want_bias = bias is not None and need[2]
        # the rounding to the dtype and the bias gradient's column sums in one pass over the accumulator
        done = _native.grad_value_finish(acc, memory.dtype, want_bias) if memory.dtype != torch.float64 else None
        if done is not None:
            gv, bias_sum = done
        else:
            gv = acc.to(memory.dtype) if memory.dtype in (torch.float16, torch.bfloat16) else acc
            bias_sum = acc.sum(0) if want_bias else None
        grad_memory = grad_weight = grad_bias = None
        if need[0]:
            grad_memory = (gv @ weight.to(gv.dtype)).view(B, N, C).to(memory.dtype)
        if need[1]:
            grad_weight = (gv.t() @ memory.reshape(B * N, C).to(gv.dtype)).to(weight.dtype)
        if want_bias:
            grad_bias = bias_sum.to(bias.dtype)
        return (grad_memory, grad_weight, grad_bias, None, None, grad_loc if need[5] else None,
                grad_attn if need[6] else None, None, None)


def ma_deform_attn_train(memory, value_weight, value_bias, spatial_shapes, level_start_index, sampling_locations,
                         attention_weights, mode, value_padding_mask=None):
    """The differentiable CUDA call (mode 'fused' or 'project' for the forward)."""
    mask = _native.check_mask(value_padding_mask, memory)
    return MaDeformAttnFunction.apply(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                      sampling_locations, attention_weights, mode, mask)
