"""ctypes bindings of the engine's C ABI (include/xse_emb.h).

The shared library libxse_emb.so is built in-tree (see Makefile). Loading it is
mandatory: there is no CPU fallback, so a missing or unloadable library raises
ImportError at import time.
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libxse_emb.so")

# absl::StatusCode numbering.
OK = 0
CANCELLED = 1
UNKNOWN = 2
INVALID_ARGUMENT = 3
DEADLINE_EXCEEDED = 4
NOT_FOUND = 5
ALREADY_EXISTS = 6
RESOURCE_EXHAUSTED = 8
FAILED_PRECONDITION = 9
UNIMPLEMENTED = 12
INTERNAL = 13

STATUS_NAMES = {
    OK: "OK",
    CANCELLED: "CANCELLED",
    UNKNOWN: "UNKNOWN",
    INVALID_ARGUMENT: "INVALID_ARGUMENT",
    DEADLINE_EXCEEDED: "DEADLINE_EXCEEDED",
    NOT_FOUND: "NOT_FOUND",
    ALREADY_EXISTS: "ALREADY_EXISTS",
    RESOURCE_EXHAUSTED: "RESOURCE_EXHAUSTED",
    FAILED_PRECONDITION: "FAILED_PRECONDITION",
    UNIMPLEMENTED: "UNIMPLEMENTED",
    INTERNAL: "INTERNAL",
}

DT_F32, DT_BF16, DT_I8_ROWWISE = 0, 1, 2
COMBINE_SUM, COMBINE_MEAN, COMBINE_SQRTN = 1, 2, 3
INDEX_I32, INDEX_I64 = 0, 1
PLACE_COPY_FROM_HOST, PLACE_COPY_FROM_DEVICE, PLACE_ADOPT_DEVICE = 0, 1, 2
EXEC_STRICT, EXEC_FUSED, EXEC_ASYNC = 0, 1, 2

COMBINE_MODES = {"SUM": COMBINE_SUM, "MEAN": COMBINE_MEAN,
                 "SQRT_N": COMBINE_SQRTN, "SQRTN": COMBINE_SQRTN}


class XseError(RuntimeError):
  """A non-OK status returned through the C ABI."""

  def __init__(self, code, message):
    super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")
    self.code = code
    self.message = message


class EngineOptions(ctypes.Structure):
  _fields_ = [("device", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class TableDesc(ctypes.Structure):
  _fields_ = [
      ("name", ctypes.c_char_p),
      ("dtype", ctypes.c_int32),
      ("combine", ctypes.c_int32),
      ("vocab", ctypes.c_int64),
      ("dim", ctypes.c_int32),
      ("placement", ctypes.c_int32),
      ("rows", ctypes.c_void_p),
      ("scale", ctypes.c_void_p),
      ("bias", ctypes.c_void_p),
      ("row_begin", ctypes.c_int64),
      ("row_end", ctypes.c_int64),
  ]


class TableInfo(ctypes.Structure):
  _fields_ = [
      ("dtype", ctypes.c_int32),
      ("combine", ctypes.c_int32),
      ("dim", ctypes.c_int32),
      ("reserved", ctypes.c_int32),
      ("vocab", ctypes.c_int64),
      ("row_begin", ctypes.c_int64),
      ("row_end", ctypes.c_int64),
      ("rows", ctypes.c_void_p),
  ]


class BagRequest(ctypes.Structure):
  _fields_ = [
      ("feature_name", ctypes.c_char_p),
      ("ids", ctypes.c_void_p),
      ("ids_type", ctypes.c_int32),
      ("offsets_type", ctypes.c_int32),
      ("num_ids", ctypes.c_int64),
      ("offsets", ctypes.c_void_p),
      ("num_offsets", ctypes.c_int64),
      ("weights", ctypes.c_void_p),
      ("num_weights", ctypes.c_int64),
      ("output", ctypes.c_void_p),
      ("output_stride", ctypes.c_int64),
  ]


_I = ctypes.c_int
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64

# name -> (restype, argtypes); every entry point declared in include/xse_emb.h.
SIGNATURES = {
    "xse_last_error": (ctypes.c_char_p, []),
    "xse_abi_version": (_I32, []),
    "xse_last_launch_count": (_I32, []),
    "xse_engine_create": (_I, [ctypes.POINTER(EngineOptions), _P]),
    "xse_engine_destroy": (None, [_P]),
    "xse_engine_add_table": (_I, [_P, ctypes.POINTER(TableDesc)]),
    "xse_engine_register_feature": (_I, [_P, ctypes.c_char_p, ctypes.c_char_p,
                                         _I32]),
    "xse_engine_clear": (_I, [_P]),
    "xse_engine_table_info": (_I, [_P, ctypes.c_char_p,
                                   ctypes.POINTER(TableInfo)]),
    "xse_engine_feature_table": (_I, [_P, ctypes.c_char_p, ctypes.c_char_p,
                                      _I32, ctypes.POINTER(_I32)]),
    "xse_status_create": (_I, [_I32, _P]),
    "xse_status_destroy": (None, [_P]),
    "xse_engine_execute_batch": (_I, [_P, ctypes.POINTER(BagRequest), _I32, _P,
                                      _I32, _P]),
    "xse_status_wait": (_I, [_P, _P]),
    "xse_engine_execute_batch_noalloc": (_I, [_P, ctypes.POINTER(BagRequest),
                                              _I32, _P]),
    "xse_engine_execute_legacy": (_I, [_P, ctypes.POINTER(BagRequest), _I32,
                                       _P]),
    "xse_engine_set_profiling": (_I, [_P, _I32]),
    "xse_engine_profile_read": (_I, [_P, ctypes.POINTER(ctypes.c_double),
                                     ctypes.POINTER(_I64),
                                     ctypes.POINTER(_I64)]),
    "xse_engine_profile_read_stages": (_I, [
        _P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_I64),
        ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_I64),
        ctypes.POINTER(_I64)]),
    "xse_engine_execute_interaction": (_I, [_P, _P, _I32, _P, _I64, _I64, _P,
                                            _I64, _P, _I32, _P]),
    "xse_engine_execute_interaction_tf32": (_I, [_P, _P, _I32, _P, _I64,
                                                 _I64, _P, _P, _I64, _P,
                                                 _I32, _P]),
    "xse_dot_interaction": (_I, [_P, _P, _I64, _I32, _I32, _P, _P]),
    "xse_synth_table": (_I, [_P, _P, _P, _I32, _U64, _U64, _I64, _I64, _I32,
                             _P]),
    "xse_synth_lengths": (_I, [_P, _I64, _I32, _I32, _U64, _U64, _P]),
    "xse_synth_ids": (_I, [_P, _I64, _I64, ctypes.c_double, _U64, _U64, _U64,
                           _U64, _I64, _P]),
    "xse_synth_weights": (_I, [_P, _I64, _U64, _U64, _I64, _P]),
}


HB_INVALID, HB_S32, HB_S64, HB_F32 = 0, 1, 2, 3
HB_MAX_RANK = 8


SHARD_NONE, SHARD_TABLEWISE, SHARD_ROWWISE = 0, 1, 2


class LoadOptions(ctypes.Structure):
  """xse_load_options (include/xse_ops.h)."""
  _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
              ("sharding", ctypes.c_int32),
              ("upload_threads", ctypes.c_int32),
              ("chunk_bytes", ctypes.c_int64)]


class HostBufferStruct(ctypes.Structure):
  _fields_ = [
      ("data", ctypes.c_void_p),
      ("dtype", ctypes.c_int32),
      ("rank", ctypes.c_int32),
      ("dims", ctypes.c_int64 * HB_MAX_RANK),
  ]


_HBP = ctypes.POINTER(HostBufferStruct)
_STRS = ctypes.POINTER(ctypes.c_char_p)

# Operator layer (include/xse_ops.h).
SIGNATURES.update({
    "xse_host_buffer_alloc": (_I, [_I32, _I32, ctypes.POINTER(_I64), _HBP]),
    "xse_host_buffer_free": (None, [_HBP]),
    "xse_resource_load": (_I, [_STRS, _STRS, _I32, _I32, _P]),
    "xse_resource_load_sharded": (_I, [_STRS, _STRS, _I32, _I32,
                                       ctypes.POINTER(LoadOptions), _P]),
    "xse_resource_create": (_I, [_I32, _P]),
    "xse_resource_destroy": (None, [_P]),
    "xse_resource_engine": (_P, [_P]),
    "xse_resource_embedding_dim": (_I, [_P, ctypes.c_char_p,
                                        ctypes.POINTER(_I32)]),
    "xse_resource_register_embedding_dim": (_I, [_P, ctypes.c_char_p, _I32]),
    "xse_lookup_transform_create": (_I, [_P, _STRS, _I32, _I32, _STRS, _I32,
                                         _I64, _P]),
    "xse_lookup_transform_destroy": (None, [_P]),
    "xse_lookup_transform_run": (_I, [_P, _HBP, _I32, _HBP, _I32, _HBP, _I32,
                                      _HBP, _P]),
    "xse_dense_lookup_transform_create": (_I, [_P, _STRS, _I32, _I64, _STRS,
                                               _I32, _P]),
    "xse_dense_lookup_transform_destroy": (None, [_P]),
    "xse_dense_lookup_transform_run": (_I, [_P, _HBP, _I32, _HBP, _P]),
})


# DLRM dense tower (include/xse_dlrm.h).
ACT_NONE, ACT_RELU, ACT_SIGMOID = 0, 1, 2
MATH_FP32, MATH_BF16X9, MATH_TF32 = 0, 1, 2
SIGNATURES.update({
    "xse_linear_forward": (_I, [_P, _I64, _I32, _I64, _P, _P, _I32, _I32,
                                _I32, _P, _I64, _P]),
    "xse_dot_interaction_strided": (_I, [_P, _I64, _P, _I64, _I64, _I32, _I32,
                                         _P, _I64, _P]),
    "xse_tf32_split": (_I, [_P, _I64, _I32, _I64, _P, _P, _P]),
    "xse_linear_forward_tf32x3": (_I, [_P, _P, _I64, _I32, _I64, _P, _P, _P,
                                       _I32, _I32, _P, _I64, _P]),
})


# Peer-memory exchange (include/xse_peer.h).
PEER_MAX_RANKS = 8


class IpcHandle(ctypes.Structure):
  _fields_ = [("bytes", ctypes.c_ubyte * 64)]


SIGNATURES.update({
    "xse_peer_group_create": (_I, [_I32, _I32, _I32, _I64, _P,
                                   ctypes.POINTER(IpcHandle)]),
    "xse_peer_group_connect": (_I, [_P, ctypes.POINTER(IpcHandle), _I32]),
    "xse_peer_group_buffer": (_P, [_P, _I32]),
    "xse_peer_group_barrier": (_I, [_P, _I64, _P]),
    "xse_peer_group_check": (_I, [_P, _P]),
    "xse_peer_group_destroy": (None, [_P]),
})


class CsrSegment(ctypes.Structure):
  """xse_csr_segment (include/xse_shard.h)."""
  _fields_ = [
      ("ids", ctypes.c_void_p),
      ("offsets", ctypes.c_void_p),
      ("weights", ctypes.c_void_p),
      ("num_ids", ctypes.c_int64),
      ("num_bags", ctypes.c_int64),
      ("ids_type", ctypes.c_int32),
      ("offsets_type", ctypes.c_int32),
      ("dst_ids", ctypes.c_void_p),
      ("dst_offsets", ctypes.c_void_p),
      ("dst_weights", ctypes.c_void_p),
      ("dst_base", ctypes.c_int64),
  ]


SIGNATURES.update({
    "xse_csr_extents": (_I, [ctypes.POINTER(CsrSegment), _I32, _P, _P]),
    "xse_csr_pack": (_I, [ctypes.POINTER(CsrSegment), _I32, _P]),
})

# Sharded execution (include/xse_shard.h).
SHARD_ID_BYTES = 128
SHARD_TABLE_PEER, SHARD_TABLE_A2A, SHARD_TABLE_PIPELINED, SHARD_ROW = 0, 1, 2, 3
SHARD_DEFER_WAIT = 1


class ShardPlanStruct(ctypes.Structure):
  """xse_shard_plan (include/xse_shard.h)."""
  _fields_ = [
      ("mode", ctypes.c_int32),
      ("num_tables", ctypes.c_int32),
      ("dim", ctypes.c_int32),
      ("chunks", ctypes.c_int32),
      ("batch", ctypes.c_int64),
      ("spin_limit", ctypes.c_int64),
  ]


SIGNATURES.update({
    "xse_shard_unique_id": (_I, [ctypes.c_char_p]),
    "xse_shard_comm_create": (_I, [_I32, _I32, _I32, ctypes.c_char_p, _P]),
    "xse_shard_comm_adopt": (_I, [_P, _I32, _I32, _I32, _P]),
    "xse_shard_comm_abort": (_I, [_P]),
    "xse_shard_comm_destroy": (None, [_P]),
    "xse_shard_exchange_create": (_I, [_P, _P, ctypes.POINTER(ShardPlanStruct),
                                       _P]),
    "xse_shard_exchange_run": (_I, [_P, ctypes.POINTER(BagRequest), _I32,
                                    _I32, _P, _P]),
    "xse_shard_exchange_ready": (_I, [_P, _P]),
    "xse_shard_exchange_check": (_I, [_P, _P]),
    "xse_shard_exchange_destroy": (None, [_P]),
})


def _load():
  if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `make -C {_HERE}` "
        "(the engine has no CPU fallback)")
  lib = ctypes.CDLL(LIB_PATH)
  for name, (restype, argtypes) in SIGNATURES.items():
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = argtypes
  return lib


lib = _load()


def last_error():
  msg = lib.xse_last_error()
  return msg.decode() if msg else ""


def check(rc):
  """Raises XseError for a non-OK status code."""
  if rc != OK:
    raise XseError(rc, last_error())
  return rc
