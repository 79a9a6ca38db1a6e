"""B200-native (sm_100a) WANferenz MoE decode path.

* ``wanferenz_b200.ops``  - the reference operator API (act_quant, fp8_gemm, fp4_gemm, ...)
* ``wanferenz_b200.moe``  - ``MoELayer`` and the ``install`` / ``bank_layout`` drop-in
* ``wanferenz_b200.ep``   - expert parallelism over torch.distributed (NCCL)

All compute runs in ``lib/libwfb200.so`` (C ABI in ``include/wfb200.h``).
"""

from ._lib import WfError, load  # noqa: F401

__all__ = ["load", "WfError"]
