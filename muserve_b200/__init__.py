"""B200-native (sm_100a) FP8 mixture-of-experts path of muserve.

The compute path is the CUDA library ``libmuserve_moe.so`` (C ABI in
``include/muserve_moe.h``); the Python modules mirror the reference's operator signatures:

* ``muserve_b200.model.qwen35_layer_v2.moe_forward``   <- muserve/model/qwen35_layer_v2.py:561
* ``muserve_b200.kernels.moe_dispatch.moe_gate / moe_experts_fp8``  <- muserve/kernels/moe_dispatch.py
* ``muserve_b200.kernels.batched_moe.batched_moe_forward``          <- muserve/kernels/batched_moe.py
* ``muserve_b200.kernels.fp8_matmul.w8a8_block_fp8_matmul``          <- muserve/kernels/fp8_matmul.py
* ``muserve_b200.mate.gemm.ragged_m_moe_gemm_8bit / gemm_fp8_nt_groupwise`` <- the mate ops
* ``muserve_b200.distributed.all_reduce``                            <- muserve/distributed.py:62
"""
__version__ = "0.1.0"
