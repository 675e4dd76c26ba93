"""Parallel training entry points.

  dp            data parallel (the GPT-2 trainer: bucketed gradient all-reduce
                overlapped with backward, CUDA graph)
  ddp           data parallel wrapper for any module (bucketed all-reduce
                overlapping backward)
  zero          sharded data parallel optimizer (ZeRO stage 1: optimizer state) for any module
  tensor        tensor parallel SwiGLU MLP step (fused all-gather -> GEMM and
                GEMM -> reduce-scatter, forward and backward)
  expert        expert parallel MoE step (fused dispatch / combine, forward and
                backward)
  sequence      Ulysses sequence parallelism (all-to-all around head-sharded
                attention)
  context       ring attention (context parallelism)
  pipeline      1F1B pipeline schedule over point-to-point transfers
  hierarchical  the two-level node x cross-node communicator
"""
