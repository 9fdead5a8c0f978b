"""``fuseop`` under its own name: the FuseSampleAgg Python API
(fuseop/__init__.py:75-214) served by this repository's B200 kernels.

Code written against the reference keeps ``import fuseop`` /
``from fuseop import fused_sample_agg_2hop`` unchanged once this
repository's root is on ``sys.path``.  The four functions are those of
``fusesampleagg_b200`` (same arguments, defaults, return containers,
autograd replay and errors; plus the keyword-only ``batch_offset``).  Like
the reference (fuseop/__init__.py:7-12), the import fails when the native
extension is not built -- there is no fallback.
"""

from __future__ import annotations

from fusesampleagg_b200 import (
    fused_sample_agg,
    fused_sample_agg_2hop,
    fused_sample_agg_2hop_with_samples,
    fused_sample_agg_with_samples,
)

__all__ = [
    "fused_sample_agg",
    "fused_sample_agg_with_samples",
    "fused_sample_agg_2hop",
    "fused_sample_agg_2hop_with_samples",
]
