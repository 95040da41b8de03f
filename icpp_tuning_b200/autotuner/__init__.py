"""Autotuner: descriptor API, cost models, search space and GPU spec.

Mirrors kernel/autotuner/ of the reference (its __init__.py:1-26 re-exports the
descriptor API).  The "LightGBM residual" and "decision table" that the reference's
package docstring announces are not implemented there either.
"""
from .interface import (  # noqa: F401
    TileLangKernelBase,
    configure_autotuner_cache,
    rank_all,
    select_best,
)
