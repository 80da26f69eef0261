"""Core-attention disaggregation (CAD): a second serving mode in which *attention GPUs* keep
only the KV cache and run the decode attention kernel, while *model GPUs* run everything
else (projections, norms, router, experts, sampling). See :mod:`fastafd_b200.cad.runtime`.
Reference: python/minisgl/cad/*.py, python/minisgl/kernel/cad_hop.py."""
