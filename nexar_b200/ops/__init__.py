"""Model-side kernels (sm_100a) with autograd wrappers."""
from .functional import (  # noqa: F401
    cross_entropy, cross_entropy_loss_only, embedding, gelu, layer_norm,
    residual_layer_norm, swiglu,
)
