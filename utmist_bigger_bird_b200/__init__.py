"""B200-native (sm_100a) Bigger Bird v3 sparse prefill attention.

Drop-in surfaces of the reference project (derkychen/utmist-bigger-bird):
  * ``bigger_bird_flash``   -- kernels/bigger_bird_flash.py
  * ``RDAttention``, ``install``, ``rope_inplace``, ``vertical_budget`` -- modal_rd/attention.py
  * ``bigger_bird_decode``, ``bigger_bird_route`` -- kernels/bigger_bird_decode.py, bigger_bird_route.py
  * ``install_chunked_mlp``, ``install_cpu_embedding``, ``install_inplace_residual`` -- the
    whole-model memory savers of modal_rd/{mlp_chunk,cpu_embed,inplace_residual}.py
The compute runs in ``libbb_b200.so`` (C ABI: include/bb_b200.h); build it with
``python -m utmist_bigger_bird_b200.build``.
"""
from .attention import RDAttention, forward_pool, install, rope_inplace, vertical_budget  # noqa: F401
from .bigger_bird_flash import bigger_bird_flash  # noqa: F401
from .bigger_bird_decode import bigger_bird_decode  # noqa: F401
from .bigger_bird_route import bigger_bird_route, pooled_probs  # noqa: F401
from .cpu_embed import CPUEmbedding, install_cpu_embedding  # noqa: F401
from .inplace_residual import install_inplace_residual  # noqa: F401
from .mlp_chunk import install_chunked_mlp  # noqa: F401
from .rmsnorm import install_fused_rmsnorm  # noqa: F401

__all__ = ["RDAttention", "install", "rope_inplace", "vertical_budget", "forward_pool", "bigger_bird_flash",
           "bigger_bird_decode", "bigger_bird_route", "pooled_probs", "CPUEmbedding", "install_cpu_embedding",
           "install_inplace_residual", "install_chunked_mlp", "install_fused_rmsnorm"]
