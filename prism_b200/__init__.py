"""prism_b200 -- B200-native (sm_100a) dynamic block-shape block-sparse
attention for Tencent-Hunyuan/Prism's video self-attention.

Public entry points mirror the reference names:
  flash_attn_bsa_3d_dynamic   hymm/models/modules/block_sparse_attention/dynamic_block_attention.py:194
  run_bsa_dynamic             SelfAttention._run_bsa_dynamic, wan_video_dit.py:342
  flash_attn_bsa_3d           block_sparse_attention/bsa_interface.py:1123 (uniform chunks)
  run_bsa_uniform             the uniform dispatch of SelfAttention, wan_video_dit.py:470-560
  flash_attn_bsa_3d_variance_guided / flash_attn_bsa_3d_audio_guided
                              block_sparse_attention/bsa_interface.py:1179, 1395 (guided selection)
  compute_channel_variance_density, compute_block_audio_saliency,
  audio_weighted_mean_pooling_compression, compute_audio_spatial_concentration_gate,
  compute_timestep_reliability_gate   bsa_interface.py:831-1102 (guidance statistics)
  flash_attn_bsa_cross        block_sparse_attention/bsa_interface.py:1276 (3D / 1D cross-modal)
  bsa_rectified_sparse_attn / bsa_taylor_sparse_attn
                              block_sparse_attention/bias_rectification.py:380, 261 (inference)
  select_zone_shapes          block_sparse_attention/dynamic_block_shape.py:358
  all_to_all_4D / all_gather  hymm/utils/communications.py:277, 401
The kernels live in libprism_bsa.so (C ABI: include/prism_bsa.h).
"""
from .bias_rectification import bsa_rectified_sparse_attn, bsa_taylor_sparse_attn  # noqa: F401
from .bsa_interface import (  # noqa: F401
    flash_attn_bsa_3d, flash_attn_bsa_3d_audio_guided, flash_attn_bsa_3d_variance_guided,
    flash_attn_bsa_cross, run_bsa_uniform,
)
from .guidance import (  # noqa: F401
    audio_weighted_mean_pooling_compression, compute_audio_spatial_concentration_gate,
    compute_block_audio_saliency, compute_channel_variance_density,
    compute_timestep_reliability_gate,
)
from .dynamic_block_attention import build_plan, flash_attn_bsa_3d_dynamic, run_bsa_dynamic  # noqa: F401
from .dynamic_block_shape import (  # noqa: F401
    ALL_CANDIDATE_SHAPES, CANDIDATE_SHAPES_64, CANDIDATE_SHAPES_128, NUM_CANDIDATES,
    NUM_CANDIDATES_64, ZONE_SIZE, compute_effective_gradient, select_zone_shapes,
)
from .ops import token_norms  # noqa: F401

__version__ = "0.1.0"
