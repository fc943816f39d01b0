"""Import name of upstream marearts-tinydeform, served by the B200 implementation.

Code written against upstream (``from marearts_tinydeform import ma_deform_attn``) runs unchanged: every public
name and the module attributes upstream's tests read (FUSED_LIMIT, FUSED_LIMIT_SM75, _limits, MODES, __version__)
are the objects of ``marearts_tinydeform_b200``.
"""

from marearts_tinydeform_b200 import (FUSED_LIMIT, FUSED_LIMIT_SM75, FUSED_LIMIT_SM100, MODES, __version__,
                                      _limits, choose_mode, ma_deform_attn, ma_deform_attn_reference)

__all__ = ['ma_deform_attn', 'ma_deform_attn_reference', 'choose_mode']
