"""Loader-level entry points mirroring the reference's ``src/kops/registry/<slug>.py``.

Each module exposes ``kernel(...)`` (and ``decode_kernel(...)`` where the reference has
one) with the same arguments, so it drops into the reference's ``Config.custom`` and
``modeling.swaps._experts_fwd`` call sites.
"""
