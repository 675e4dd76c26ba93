"""Parallel training entry points: data (dp), tensor (tp) and expert (ep)
parallel, and the two-level node x cross-node communicator (hierarchical)."""
