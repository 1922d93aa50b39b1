"""B200 (sm_100a) implementation of the MiniMind-mHC residual path.

Same module layout as the reference project's ``model`` package for the mHC
files: ``mhc_common`` (StreamExpand, MHCHead), ``mhc_fused``
(MHCConnection_Fused, sinkhorn_normalize) and ``mhc_fused_no_hres``
(MHCConnection_FusedNoHres).  The kernels live in ``libmhc_b200.so`` next to
this file (C ABI: ``include/mhc_b200.h``).
"""
