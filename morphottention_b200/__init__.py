"""B200 (sm_100a) MorphoAttention: drop-in for the reference ``morphottention`` package.

``MorphoAttention``, ``MorphoAttentionFunction`` and ``morpho_attention`` keep the
reference's signatures and call ``torch.ops.morphottention.forward/backward``, which are
backed by hand-written tcgen05/TMA kernels behind the C ABI in ``include/morpho_sm100.h``.
"""

from .autograd import (MorphoAttention, MorphoAttentionFunction, SoftMorphAttention, SoftMorphAttentionFunction,
                       attention_options, get_cube_projection, get_grad_mode, get_mask_diag, get_score, grad_mode,
                       morpho_attention, set_cube_projection, set_grad_mode, set_mask_diag, set_score,
                       soft_morph_attention)

__all__ = ["MorphoAttention", "MorphoAttentionFunction", "morpho_attention", "set_grad_mode", "get_grad_mode",
           "grad_mode", "set_cube_projection", "get_cube_projection", "set_mask_diag", "get_mask_diag",
           "set_score", "get_score", "attention_options", "SoftMorphAttention", "SoftMorphAttentionFunction",
           "soft_morph_attention"]
