"""B200-native block-sparse attention engine behind the longcat_video BSA API.

Import paths mirror xocialize/longcat-video-mlx (``longcat_video.models.block_sparse_attention``
and friends) so the engine can replace the MLX modules in place.
"""

__version__ = "0.1.0"
