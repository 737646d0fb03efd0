"""B200-native embedding-bag and DLRM interaction engine.

Drop-in GPU engine for the CPU embedding path of openxla/xla-serving
(data/cpu_embedding/cc and data/kernels/cpu_embedding). Host code calls
hand-written sm_100a CUDA kernels through the C ABI in include/xse_emb.h;
this package binds that ABI. There is no CPU fallback: importing the package
fails if the CUDA library is missing.
"""

from . import _capi
from . import dlrm
from . import ops
from . import sharding
from ._capi import XseError
from .engine import (BagRequest, EmbeddingEngine, PreparedBatch, Status,
                     dot_interaction, last_launch_count, stream_handle)

__all__ = [
    "BagRequest", "EmbeddingEngine", "PreparedBatch", "Status", "XseError",
    "dot_interaction", "last_launch_count", "stream_handle",
]
