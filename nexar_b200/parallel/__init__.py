"""Parallel training entry points: data (dp), tensor (tp) and expert (ep) parallel."""
