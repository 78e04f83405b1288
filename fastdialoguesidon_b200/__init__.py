"""fastdialoguesidon_b200: the FastDialogueSidon attention hot path on B200.

Public API (mirrors the attention ops of ``fds_triton.kernels``):

- :func:`flexrel_attention` / :func:`flexrel_attention_split` /
  :func:`encoder_attention`: w2v-BERT relative_key self-attention;
  :func:`flexrel_attention_qr`: the same with q, k, v and q.rel^T given
  separately, in the TensorRT plugin's [B, L, H, D] layout;
- :func:`rope_attention`: the DiT head's RoPE self-attention (replaces
  ``rope_split`` + SDPA), and :func:`rope_split` itself;
- :func:`linear` / :func:`linear_rope` / :func:`accumulate`: the projections
  either side of the attention (QKV with bias, the DiT's QKV with RoPE in the
  epilogue, the out-projection accumulated into the fp32 residual), and
  :func:`rotated_attention` for the DiT attention over a pre-rotated qkv;
- :func:`check_status`: raise if a kernel reported a bounded-wait timeout.

The same ops are registered as ``torch.ops.fds.flexrel_attention`` and
``torch.ops.fds.rope_attention`` (see :mod:`.torch_ops`).
"""

from .kernels import (  # noqa: F401
    LEFT,
    NUM_POS,
    NUM_POS_PAD,
    RIGHT,
    FdsError,
    accumulate,
    check_status,
    cudnn_attention_available,
    encoder_attention,
    flexrel_attention,
    flexrel_attention_qr,
    flexrel_attention_split,
    linear,
    linear_rope,
    rope_attention,
    rope_split,
    rope_tables,
    rotated_attention,
)
from . import torch_ops  # noqa: F401  (registers torch.ops.fds.*)

__version__ = "0.1.0"
