"""Model-side kernels (sm_100a) with autograd wrappers."""
from .functional import (  # noqa: F401
    colsum, cross_entropy, cross_entropy_loss_only, embedding, gelu, layer_norm, linear, matmul_nt,
    residual_layer_norm, swiglu,
)
