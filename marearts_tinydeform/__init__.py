"""Import name of upstream marearts-tinydeform, served by the B200 implementation.

Code written against upstream (``from marearts_tinydeform import ma_deform_attn``) runs unchanged: every public
name and the module attributes upstream's tests read (FUSED_LIMIT, FUSED_LIMIT_SM75, _limits, MODES, __version__)
are the objects of ``marearts_tinydeform_b200``, and ``ma_deform_attn`` keeps upstream's contract to the letter,
its inference-only rule included (``marearts_tinydeform/__init__.py:49-79`` upstream): CUDA inputs that require
grad are rejected with upstream's RuntimeError. Training goes through the B200 package's own name,
``marearts_tinydeform_b200.ma_deform_attn``, which differentiates.
"""

import torch

import marearts_tinydeform_b200 as _b200
from marearts_tinydeform_b200 import (FUSED_LIMIT, FUSED_LIMIT_SM75, FUSED_LIMIT_SM100, MODES, __version__,
                                      _limits, choose_mode, ma_deform_attn_reference)

__all__ = ['ma_deform_attn', 'ma_deform_attn_reference', 'choose_mode']


def ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                   sampling_locations, attention_weights, mode='auto'):
    """value = memory @ value_weight.T + value_bias, then multi-scale deformable attention; [B, Q, H * D].

    Upstream's signature and checks, in upstream's order: an unknown mode raises ValueError; CPU tensors run
    ma_deform_attn_reference; CUDA tensors need the native library (RuntimeError without it); inputs that require
    grad while grad mode is on raise RuntimeError (inference only); then the B200 kernels run the order `mode`
    names ('auto' picks one with choose_mode).
    """
    if mode not in MODES:
        raise ValueError(f'mode must be one of {MODES}, got {mode!r}')
    if not memory.is_cuda:
        return ma_deform_attn_reference(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                        sampling_locations, attention_weights)
    _b200._native.load()  # RuntimeError when the CUDA library is missing: there is no fallback
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad
            for t in (memory, value_weight, value_bias, sampling_locations, attention_weights)):
        raise RuntimeError('ma_deform_attn is inference only: run it under torch.no_grad() / '
                           'torch.inference_mode(), or use ma_deform_attn_reference for training')
    return _b200.ma_deform_attn(memory, value_weight, value_bias, spatial_shapes, level_start_index,
                                sampling_locations, attention_weights, mode=mode)
