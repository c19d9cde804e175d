"""Hot ops: the public API (``api``), the fp32 oracle (``reference``) and the sm_100a kernels."""
