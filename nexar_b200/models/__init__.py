"""Model families driven by the nexar_b200 kernels."""
from .gpt2 import GPT2, GPT2Config  # noqa: F401
