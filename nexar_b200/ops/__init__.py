"""Model-side kernels (sm_100a) with autograd wrappers."""
from .functional import (  # noqa: F401
    attention, attention_supported, colsum, cross_entropy, cross_entropy_loss_only, embedding, gelu, layer_norm,
    linear, matmul_fp8, matmul_nt, quant_fp8_128x128, quant_fp8_1x128,
    residual_layer_norm, swiglu, swiglu_quant_fp8,
)
