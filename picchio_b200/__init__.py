"""picchio_b200: picchio's per-token MoE hot path on B200 (sm_100a).

The compute lives in ``libpicchio_b200.so`` (CUDA kernels behind the C ABI of
``include/picchio_b200.h``); this package is the Python mirror of the
reference's interface over that ABI (ctypes).  There is no CPU path: if the
library is missing or no CUDA device is present, calls raise.
"""
from .api import (  # noqa: F401
    PicchioError, Model, ModelConfig, QT, nccl_unique_id, lib, LIB_PATH,
    FMT_F32, FMT_INT8, FMT_INT4, FMT_MXFP4,
)
