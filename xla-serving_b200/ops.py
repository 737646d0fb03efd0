"""Host-buffer operators and the table resource (C ABI: include/xse_ops.h).

Python surface of the operator layer, mirroring the reference's
`CpuEmbeddingResource` (data/kernels/cpu_embedding/cpu_embedding_module.py:
114-296) and the `CpuEmbeddingLookupTransform` /
`DenseCpuEmbeddingLookupTransform` operators (cpu_embedding_lookup_transform.h,
dense_cpu_embedding_lookup_transform.h). Inputs and outputs are numpy arrays
(host buffers); the work runs in the engine's CUDA kernels.
"""

import ctypes
import os
import tempfile
from typing import Dict, List, Optional, Sequence, Union

import numpy as np

from . import _capi as C
from .engine import EmbeddingEngine, stream_handle

MANIFEST_ASSET_NAME = "__jce_manifest__"

_NP_TO_HB = {np.dtype(np.int32): C.HB_S32, np.dtype(np.int64): C.HB_S64,
             np.dtype(np.float32): C.HB_F32}
_HB_TO_NP = {C.HB_S32: np.int32, C.HB_S64: np.int64, C.HB_F32: np.float32}


class HostBuffer:
  """A numpy array viewed as an XSE host buffer (kept alive while in use).

  `HostBuffer.empty()` is the uninitialized buffer ("Empty host buffer");
  `dtype_code` overrides the element type code for negative tests.
  """

  def __init__(self, array=None, dtype_code=None, data_ptr=None, shape=None):
    self.struct = C.HostBufferStruct()
    self.array = None
    if array is None and data_ptr is None:
      self.struct.dtype = C.HB_INVALID
      return
    if array is not None:
      array = np.asarray(array)
      if not array.flags.c_contiguous:  # (ascontiguousarray would make a
        array = array.copy(order="C")   # 0-d array 1-d)
      self.array = array
      shape = array.shape
      data_ptr = array.ctypes.data if array.size else None
      code = _NP_TO_HB.get(array.dtype, 99)
    else:
      code = C.HB_S64
    self.struct.data = data_ptr
    self.struct.dtype = code if dtype_code is None else dtype_code
    self.struct.rank = len(shape)
    for i, d in enumerate(shape):
      self.struct.dims[i] = d

  @staticmethod
  def empty():
    return HostBuffer()


def _as_buffer(x):
  return x if isinstance(x, HostBuffer) else HostBuffer(x)


def _buffer_array(items):
  bufs = [_as_buffer(x) for x in items]
  arr = (C.HostBufferStruct * max(len(bufs), 1))()
  for i, b in enumerate(bufs):
    arr[i] = b.struct
  return arr, bufs


class PreparedInputs:
  """The host-buffer arrays of one operator call, converted once. Keeps the
  buffers alive; their contents may change between calls, their storage
  may not."""

  def __init__(self, ids, row_pointers=(), weights=()):
    self.ids, self._ids = _buffer_array(ids)
    self.row_pointers, self._rps = _buffer_array(row_pointers)
    self.weights, self._ws = _buffer_array(weights)
    self.num_ids = len(self._ids)
    self.num_row_pointers = len(self._rps)
    self.num_weights = len(self._ws)


class PinnedBuffer(HostBuffer):
  """A host buffer in the library's pinned memory, viewed as numpy.

  Inputs in pinned memory are copied to the device by DMA without the
  operators' host-side staging copy; operator outputs are pinned buffers.
  Free with close() (the numpy view dies with it).
  """

  def __init__(self, shape=None, dtype=np.float32, struct=None):
    # pylint: disable=super-init-not-called
    if struct is None:
      shape = tuple(int(d) for d in shape)
      struct = C.HostBufferStruct()
      dims = (ctypes.c_int64 * max(len(shape), 1))(*shape)
      C.check(C.lib.xse_host_buffer_alloc(_NP_TO_HB[np.dtype(dtype)],
                                          len(shape), dims,
                                          ctypes.byref(struct)))
    self.struct = struct
    shape = tuple(struct.dims[k] for k in range(struct.rank))
    dtype = _HB_TO_NP[struct.dtype]
    count = int(np.prod(shape)) if shape else 1
    if struct.data and count:
      raw = (ctypes.c_char * (count * np.dtype(dtype).itemsize)).from_address(
          struct.data)
      self.array = np.frombuffer(raw, dtype=dtype, count=count).reshape(shape)
    else:
      self.array = np.zeros(shape, dtype=dtype)

  def close(self):
    if self.struct is not None and self.struct.data:
      self.array = None
      C.lib.xse_host_buffer_free(ctypes.byref(self.struct))
    self.struct = None

  def __del__(self):
    try:
      self.close()
    except Exception:  # pylint: disable=broad-except
      pass


def _take_outputs(outs, n, copy=True):
  """Copies the library's pinned output buffers into numpy and frees them;
  with copy=False returns them as PinnedBuffer objects instead."""
  if not copy:
    return [PinnedBuffer(struct=C.HostBufferStruct.from_buffer_copy(outs[i]))
            for i in range(n)]
  results = []
  for i in range(n):
    o = outs[i]
    shape = tuple(o.dims[k] for k in range(o.rank))
    count = int(np.prod(shape)) if shape else 1
    if o.data and count:
      buf = (ctypes.c_float * count).from_address(o.data)
      arr = np.frombuffer(buf, dtype=np.float32, count=count).reshape(
          shape).copy()
    else:
      arr = np.zeros(shape, dtype=np.float32)
    results.append(arr)
    C.lib.xse_host_buffer_free(ctypes.byref(o))
  return results


def _names(seq):
  arr = (ctypes.c_char_p * max(len(seq), 1))()
  for i, s in enumerate(seq):
    arr[i] = s.encode()
  return arr


def _is_invalid_table_name(name):
  return (not isinstance(name, str) or not name or "/" in name or
          "\\" in name or ".." in name or name == MANIFEST_ASSET_NAME)


def _load_options(placement, upload_threads, chunk_bytes):
  opt = C.LoadOptions(1, 0, C.SHARD_NONE, int(upload_threads),
                      int(chunk_bytes))
  if placement is not None:
    kind, world, rank = placement
    kinds = {"table": C.SHARD_TABLEWISE, "row": C.SHARD_ROWWISE}
    if kind not in kinds:
      raise ValueError(f"unknown sharding {kind!r} (table or row)")
    opt.sharding, opt.world, opt.rank = kinds[kind], int(world), int(rank)
  return opt


class CpuEmbeddingResource:
  """Tables (and feature specs) loaded into HBM through the resource's asset
  format: a CpuEmbeddingManifest text proto plus one `<table>.bin` per table
  (cpu_embedding_resource.cc:51-225, cpu_embedding_serializer.cc:37-74).

  table_data: table name -> array [vocab, dim]: float32, bfloat16 bits
    (uint16) or (int8 rows, scale, bias) for int8 row-wise tables.
  combine_modes: table name -> "SUM" | "MEAN" | "SQRT_N" (default MEAN, as the
    reference's manifest builder, cpu_embedding_module.py:87).
  feature_specs: [{"name", "table_name", optional "max_sequence_length"}].
  placement: None (every table whole) or (sharding, world, rank) with
    sharding "table" (table i of the manifest on rank i mod world) or "row"
    (rows [vocab r / world, vocab (r+1) / world) of every table).
  upload_threads, chunk_bytes: the host -> HBM upload (pinned staging chunks
    filled from the asset file by that many threads; 0 = defaults,
    chunk_bytes < 0 = one pageable copy per table).
  """

  def __init__(self, table_data, combine_modes, feature_specs, *, device=0,
               max_cpu_slots=8, block_size=64, placement=None,
               upload_threads=0, chunk_bytes=0):
    self.device = device
    self._options = _load_options(placement, upload_threads, chunk_bytes)
    self._handle = ctypes.c_void_p()
    self._dir = tempfile.TemporaryDirectory(prefix="xse_assets_")
    names, paths = [MANIFEST_ASSET_NAME], []
    lines = [f"max_cpu_slots: {max_cpu_slots}", f"block_size: {block_size}"]
    for table, data in table_data.items():
      if _is_invalid_table_name(table):
        raise ValueError(
            "Invalid table name (empty, reserved, or path traversal): "
            f"{table!r}")
      path = os.path.join(self._dir.name, f"{table}.bin")
      if isinstance(data, tuple):  # int8 rows with per-row scale and bias
        q, scale, bias = data
        q = np.ascontiguousarray(q, dtype=np.int8)
        vocab, dim = q.shape
        kind = "INT8_ROWWISE"
        with open(path, "wb") as f:
          f.write(q.tobytes())
          f.write(np.ascontiguousarray(scale, np.float32).tobytes())
          f.write(np.ascontiguousarray(bias, np.float32).tobytes())
      else:
        arr = np.ascontiguousarray(data)
        vocab, dim = arr.shape
        kind = "BFLOAT16" if arr.dtype == np.uint16 else "FLOAT32"
        if kind == "FLOAT32":
          arr = arr.astype(np.float32)
        arr.tofile(path)
      mode = combine_modes.get(table, "MEAN")
      lines.append(
          f'tables {{ name: "{table}" vocab_size: {vocab} embedding_dim: '
          f'{dim} combine_mode: {mode} data_type: {kind} }}')
      names.append(table)
      paths.append(path)
    for spec in feature_specs:
      seq = spec.get("max_sequence_length", 0)
      lines.append(
          f'feature_specs {{ name: "{spec["name"]}" table: '
          f'"{spec["table_name"]}" max_sequence_length: {seq} }}')
    manifest = os.path.join(self._dir.name, "manifest.textproto")
    with open(manifest, "w", encoding="utf-8") as f:
      f.write("\n".join(lines) + "\n")
    self._load([MANIFEST_ASSET_NAME] + names[1:], [manifest] + paths)

  def _load(self, names, paths):
    C.check(C.lib.xse_resource_load_sharded(
        _names(names), _names(paths), len(names), self.device,
        ctypes.byref(self._options), ctypes.byref(self._handle)))

  @classmethod
  def from_assets(cls, assets: Dict[str, str], device=0, *, placement=None,
                  upload_threads=0, chunk_bytes=0):
    """Loads from existing asset files: {asset name: path}."""
    self = cls.__new__(cls)
    self.device = device
    self._options = _load_options(placement, upload_threads, chunk_bytes)
    self._handle = ctypes.c_void_p()
    self._dir = None
    names = list(assets)
    self._load(names, [assets[n] for n in names])
    return self

  @classmethod
  def empty(cls, device=0):
    """A resource whose engine is filled directly (tables and feature specs
    added through `engine`), as the reference's tests do."""
    self = cls.__new__(cls)
    self.device = device
    self._handle = ctypes.c_void_p()
    self._dir = None
    C.check(C.lib.xse_resource_create(device, ctypes.byref(self._handle)))
    return self

  @property
  def handle(self):
    return self._handle

  @property
  def engine(self) -> EmbeddingEngine:
    return EmbeddingEngine.borrow(C.lib.xse_resource_engine(self._handle),
                                  self.device)

  def get_embedding_dim(self, feature_name):
    dim = ctypes.c_int32()
    C.check(C.lib.xse_resource_embedding_dim(self._handle,
                                             feature_name.encode(),
                                             ctypes.byref(dim)))
    return dim.value

  def register_embedding_dim(self, feature_name, dim):
    C.check(C.lib.xse_resource_register_embedding_dim(
        self._handle, feature_name.encode(), dim))

  def close(self):
    if self._handle:
      C.lib.xse_resource_destroy(self._handle)
      self._handle = ctypes.c_void_p()
    if self._dir is not None:
      self._dir.cleanup()
      self._dir = None

  def __del__(self):
    try:
      self.close()
    except Exception:  # pylint: disable=broad-except
      pass


class CpuEmbeddingLookupTransform:
  """CSR (or dense-lookup) pooled lookups over host buffers
  (cpu_embedding_lookup_transform.h:43-56)."""

  def __init__(self, resource: CpuEmbeddingResource,
               feature_names: Union[str, Sequence[str]],
               dense_lookup: bool = False,
               output_feature_names: Optional[Sequence[str]] = None,
               embedding_dim: int = 128):
    if isinstance(feature_names, str):
      feature_names = [feature_names]
    outputs = list(output_feature_names or [])
    self.feature_names = list(feature_names)
    self._resource = resource
    self._handle = ctypes.c_void_p()
    C.check(C.lib.xse_lookup_transform_create(
        resource.handle, _names(self.feature_names), len(self.feature_names),
        1 if dense_lookup else 0, _names(outputs), len(outputs),
        embedding_dim, ctypes.byref(self._handle)))

  def __call__(self, ids, row_pointers=(), weights=(), *, stream=None,
               copy=True) -> List[np.ndarray]:
    """Pooled [batch, dim] float32 outputs, one per feature. copy=False
    returns the pinned outputs as PinnedBuffer objects (caller closes)."""
    ids_arr, keep_i = _buffer_array(ids)
    rp_arr, keep_r = _buffer_array(row_pointers)
    w_arr, keep_w = _buffer_array(weights)
    n = len(self.feature_names)
    outs = (C.HostBufferStruct * n)()
    rc = C.lib.xse_lookup_transform_run(
        self._handle, ids_arr, len(keep_i), rp_arr, len(keep_r), w_arr,
        len(keep_w), outs, stream_handle(stream))
    del keep_i, keep_r, keep_w
    C.check(rc)
    return _take_outputs(outs, n, copy)

  def run_prepared(self, prepared: "PreparedInputs", outs, *, stream=None):
    """The call with inputs converted once (a serving loop's reused host
    buffers): the pooled outputs land in `outs`, an array of
    HostBufferStruct from output_array(), as the library's pinned buffers;
    release them with free_outputs(outs) once read."""
    C.check(C.lib.xse_lookup_transform_run(
        self._handle, prepared.ids, prepared.num_ids, prepared.row_pointers,
        prepared.num_row_pointers, prepared.weights, prepared.num_weights,
        outs, stream_handle(stream)))
    return outs

  def output_array(self):
    return (C.HostBufferStruct * len(self.feature_names))()

  @staticmethod
  def free_outputs(outs):
    for o in outs:
      C.lib.xse_host_buffer_free(ctypes.byref(o))

  def close(self):
    if self._handle:
      C.lib.xse_lookup_transform_destroy(self._handle)
      self._handle = ctypes.c_void_p()

  def __del__(self):
    try:
      self.close()
    except Exception:  # pylint: disable=broad-except
      pass


class DenseCpuEmbeddingLookupTransform:
  """Dense [batch, seq] ids with pad filtering
  (dense_cpu_embedding_lookup_transform.h:37-83)."""

  def __init__(self, resource: CpuEmbeddingResource,
               feature_names: Union[str, Sequence[str]], pad_value: int = 0,
               output_feature_names: Optional[Sequence[str]] = None):
    if isinstance(feature_names, str):
      feature_names = [feature_names]
    outputs = list(output_feature_names or [])
    self.feature_names = list(feature_names)
    self.pad_value = pad_value
    self._resource = resource
    self._handle = ctypes.c_void_p()
    C.check(C.lib.xse_dense_lookup_transform_create(
        resource.handle, _names(self.feature_names), len(self.feature_names),
        pad_value, _names(outputs), len(outputs), ctypes.byref(self._handle)))

  def __call__(self, dense_ids, *, stream=None, copy=True
               ) -> List[np.ndarray]:
    if not isinstance(dense_ids, (list, tuple)):
      dense_ids = [dense_ids]
    arr, keep = _buffer_array(dense_ids)
    n = len(self.feature_names)
    outs = (C.HostBufferStruct * n)()
    rc = C.lib.xse_dense_lookup_transform_run(self._handle, arr, len(keep),
                                              outs, stream_handle(stream))
    del keep
    C.check(rc)
    return _take_outputs(outs, n, copy)

  def close(self):
    if self._handle:
      C.lib.xse_dense_lookup_transform_destroy(self._handle)
      self._handle = ctypes.c_void_p()

  def __del__(self):
    try:
      self.close()
    except Exception:  # pylint: disable=broad-except
      pass
