"""uplift_b200 -- the UPLiFT Local Attender as fused sm_100a (B200) CUDA kernels.

Drop-in for the reference's Local Attender path:
  uplift_b200.attender.LocalAttender       <- uplift/uplift.py:LocalAttender
  uplift_b200.attender.FusedLocalAttender  <- uplift/kernels/triton_attender.py:TritonLocalAttender
  uplift_b200.ops.local_attender / attender_pool  (torch custom ops)
The kernels sit behind the C ABI in include/uplift_la.h (libuplift_la.so).
"""
from .attender import FusedLocalAttender, LocalAttender, NEIGHBOURHOODS  # noqa: F401

__version__ = "0.1.0"
