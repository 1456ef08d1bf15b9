"""FlagOS_mhc on B200: the four mHC operators of liuhycs/FlagOS-mhc as
hand-written sm_100a CUDA kernels behind a C ABI (include/mhc_b200.h).

Same public names as the reference package (src/__init__.py:34-47):

    mhc_post, mhc_post_backward, mhc_pre_clamp_sinkhorn,
    mhc_pre_clamp_sinkhorn_backward          -- CUDA operators
    mhc_post_fn, mhc_pre_clamp_sinkhorn_fn,
    MhcPostFn, MhcPreClampSinkhornFn         -- autograd wrappers
    *_ref                                    -- pure-PyTorch definitions

The operators need CUDA tensors on an sm_100 GPU; there is no CPU fallback.
"""
from .mhc_post import mhc_post, mhc_post_ref
from .mhc_post_backward import mhc_post_backward, mhc_post_backward_ref
from .mhc_pre_clamp_sinkhorn import mhc_pre_clamp_sinkhorn, mhc_pre_clamp_sinkhorn_ref
from .mhc_pre_clamp_sinkhorn_backward import (mhc_pre_clamp_sinkhorn_backward,
                                              mhc_pre_clamp_sinkhorn_backward_ref)
from .autograd import MhcPostFn, MhcPreClampSinkhornFn, mhc_post_fn, mhc_pre_clamp_sinkhorn_fn

__all__ = [
    "mhc_post",
    "mhc_post_ref",
    "mhc_post_backward",
    "mhc_post_backward_ref",
    "mhc_pre_clamp_sinkhorn",
    "mhc_pre_clamp_sinkhorn_ref",
    "mhc_pre_clamp_sinkhorn_backward",
    "mhc_pre_clamp_sinkhorn_backward_ref",
    "MhcPostFn",
    "MhcPreClampSinkhornFn",
    "mhc_post_fn",
    "mhc_pre_clamp_sinkhorn_fn",
]
