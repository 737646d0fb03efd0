"""Python handle on the B200 embedding engine (C ABI in include/xse_emb.h).

Mirrors CpuEmbeddingEngine (data/cpu_embedding/cc/cpu_embedding_engine.h:
41-103) of openxla/xla-serving: tables and feature specs are registered once,
then groups of CSR lookups run in one call. Tensors are torch CUDA tensors;
torch is used only for device memory and streams, all compute runs in the
engine's CUDA kernels.
"""

import ctypes
import dataclasses
from typing import Optional, Sequence

import numpy as np
import torch

from . import _capi as C

_DTYPES = {
    torch.float32: C.DT_F32,
    torch.bfloat16: C.DT_BF16,
    torch.int8: C.DT_I8_ROWWISE,
}


def _index_type(t):
  if t.dtype == torch.int64:
    return C.INDEX_I64
  if t.dtype == torch.int32:
    return C.INDEX_I32
  raise C.XseError(C.INVALID_ARGUMENT,
                   "Embedding IDs and row pointers must be int32 or int64.")


def _ptr(t):
  return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_handle(stream=None):
  """cudaStream_t of a torch stream (the current stream by default)."""
  s = stream if stream is not None else torch.cuda.current_stream()
  return ctypes.c_void_p(s.cuda_stream)


def combine_code(combine):
  if isinstance(combine, int):
    return combine
  try:
    return C.COMBINE_MODES[combine.upper()]
  except KeyError as e:
    raise ValueError(f"Unknown combine mode: {combine}") from e


@dataclasses.dataclass
class BagRequest:
  """One feature's CSR lookup (CpuEmbeddingEngine::FeatureBatchInput,
  cpu_embedding_engine.h:55-62), on device memory."""

  feature_name: str
  ids: torch.Tensor
  offsets: torch.Tensor  # absolute CSR offsets, num_bags + 1 entries
  output: Optional[torch.Tensor]  # [num_bags, dim] or a strided view of a
                                  # wider buffer (None for
                                  # execute_interaction)
  weights: Optional[torch.Tensor] = None
  output_stride: int = 0  # floats between bags; 0 = dim


class PreparedBatch(list):
  """A group of BagRequests converted to the C request array once.

  A list of the requests (it keeps their tensors alive) that also holds
  their xse_bag_request array, so a group that runs every step -- the
  per-destination groups of a sharded exchange, a serving loop's fixed
  inputs -- skips the per-call conversion (about 3 us per request in
  Python, which at 8 tables x 8 destinations outlasts the kernels it
  launches). The tensors' storage must not change while it is in use; a
  changed list must be prepared again.
  """

  def __init__(self, requests: Sequence[BagRequest]):
    super().__init__(requests)
    self.array, self._names = EmbeddingEngine._c_requests(self)


class Status:
  """Caller-owned device status block for asynchronous execution."""

  def __init__(self, max_requests=256):
    self._handle = ctypes.c_void_p()
    C.check(C.lib.xse_status_create(max_requests, ctypes.byref(self._handle)))

  @property
  def handle(self):
    return self._handle

  def wait(self, stream=None):
    C.check(C.lib.xse_status_wait(self._handle, stream_handle(stream)))

  def close(self):
    if self._handle:
      C.lib.xse_status_destroy(self._handle)
      self._handle = ctypes.c_void_p()

  def __del__(self):
    try:
      self.close()
    except Exception:  # pylint: disable=broad-except
      pass


class EmbeddingEngine:
  """Tables in HBM plus feature specs; runs pooled lookups on the device."""

  def __init__(self, device=0):
    self.device = device
    self._handle = ctypes.c_void_p()
    self._owned = True
    opts = C.EngineOptions(device=device, reserved=0)
    C.check(C.lib.xse_engine_create(ctypes.byref(opts),
                                    ctypes.byref(self._handle)))
    self._adopted = {}  # table name -> tensors kept alive

  @classmethod
  def borrow(cls, handle, device=0):
    """A non-owning handle on an engine owned elsewhere (a resource's)."""
    self = cls.__new__(cls)
    self.device = device
    self._handle = ctypes.c_void_p(handle)
    self._owned = False
    self._adopted = {}
    return self

  def close(self):
    if self._handle and self._owned:
      C.lib.xse_engine_destroy(self._handle)
    self._handle = ctypes.c_void_p()
    self._adopted.clear()

  def __del__(self):
    try:
      self.close()
    except Exception:  # pylint: disable=broad-except
      pass

  @property
  def handle(self):
    return self._handle

  def add_table(self, name, rows, combine="SUM", *, scale=None, bias=None,
                vocab=None, row_begin=0, row_end=0, adopt=False):
    """Adds a table (EmbeddingTable::Create + AddLocalTable).

    rows: torch tensor [rows, dim] (float32, bfloat16 or int8 with per-row
      scale/bias) on the device or the host, or a numpy array (host).
    vocab: global row count when rows hold a row-wise shard
      [row_begin, row_end) of a larger table.
    adopt: borrow a device tensor instead of copying it.
    """
    keep = []
    if isinstance(rows, np.ndarray):
      if rows.dtype == np.float32:
        rows = torch.from_numpy(np.ascontiguousarray(rows))
      elif rows.dtype == np.int8:
        rows = torch.from_numpy(np.ascontiguousarray(rows))
      elif rows.dtype == np.uint16:  # bf16 bits
        rows = torch.from_numpy(
            np.ascontiguousarray(rows).view(np.int16)).view(torch.bfloat16)
      else:
        raise C.XseError(C.INVALID_ARGUMENT,
                         f"Unsupported data type: {rows.dtype}")
    if rows.dim() != 2:
      raise C.XseError(
          C.INVALID_ARGUMENT,
          "Embedding table data must be a 2D array. Got shape: "
          f"({','.join(str(d) for d in rows.shape)})")
    if rows.dtype not in _DTYPES:
      raise C.XseError(C.INVALID_ARGUMENT, f"Unsupported data type: {rows.dtype}")
    rows = rows.contiguous()
    dtype = _DTYPES[rows.dtype]
    on_device = rows.is_cuda
    placement = (C.PLACE_ADOPT_DEVICE if adopt else C.PLACE_COPY_FROM_DEVICE) \
        if on_device else C.PLACE_COPY_FROM_HOST
    if adopt and not on_device:
      raise C.XseError(C.INVALID_ARGUMENT, "Only device tables can be adopted.")
    sp = bp = None
    if dtype == C.DT_I8_ROWWISE:
      if scale is None or bias is None:
        raise C.XseError(C.INVALID_ARGUMENT,
                         "Int8 row-wise tables need per-row scale and bias.")
      scale = torch.as_tensor(scale, dtype=torch.float32)
      bias = torch.as_tensor(bias, dtype=torch.float32)
      scale = scale.to(rows.device).contiguous()
      bias = bias.to(rows.device).contiguous()
      keep += [scale, bias]
      sp, bp = scale.data_ptr(), bias.data_ptr()
    n = rows.shape[0]
    if vocab is None:
      vocab = n if row_end == 0 else row_end
    if row_begin == 0 and row_end == 0 and n != vocab:
      row_end = n
    desc = C.TableDesc(
        name=name.encode(), dtype=dtype, combine=combine_code(combine),
        vocab=vocab, dim=rows.shape[1], placement=placement,
        rows=rows.data_ptr(), scale=sp, bias=bp, row_begin=row_begin,
        row_end=row_end)
    C.check(C.lib.xse_engine_add_table(self._handle, ctypes.byref(desc)))
    if adopt:
      self._adopted[name] = [rows] + keep

  def register_feature(self, feature, table, max_sequence_length=0):
    C.check(C.lib.xse_engine_register_feature(
        self._handle, feature.encode(), table.encode(), max_sequence_length))

  def clear(self):
    C.check(C.lib.xse_engine_clear(self._handle))
    self._adopted.clear()

  def table_info(self, table):
    info = C.TableInfo()
    C.check(C.lib.xse_engine_table_info(self._handle, table.encode(),
                                        ctypes.byref(info)))
    return info

  def feature_table(self, feature):
    buf = ctypes.create_string_buffer(1024)
    seq = ctypes.c_int32()
    C.check(C.lib.xse_engine_feature_table(self._handle, feature.encode(), buf,
                                           len(buf), ctypes.byref(seq)))
    return buf.value.decode(), seq.value

  @staticmethod
  def _c_requests(requests: Sequence[BagRequest]):
    arr = (C.BagRequest * len(requests))()
    names = []
    for i, r in enumerate(requests):
      name = r.feature_name.encode()
      names.append(name)
      arr[i].feature_name = name
      arr[i].ids = None if r.ids is None else r.ids.data_ptr()
      arr[i].ids_type = C.INDEX_I64 if r.ids is None else _index_type(r.ids)
      arr[i].num_ids = 0 if r.ids is None else r.ids.numel()
      arr[i].offsets = None if r.offsets is None else r.offsets.data_ptr()
      arr[i].offsets_type = (C.INDEX_I64 if r.offsets is None
                             else _index_type(r.offsets))
      arr[i].num_offsets = 0 if r.offsets is None else r.offsets.numel()
      arr[i].weights = None if r.weights is None else r.weights.data_ptr()
      arr[i].num_weights = 0 if r.weights is None else r.weights.numel()
      arr[i].output = None if r.output is None else r.output.data_ptr()
      arr[i].output_stride = r.output_stride
    return arr, names

  def execute_batch(self, requests: Sequence[BagRequest], *, stream=None,
                    fused=False, status: Optional[Status] = None):
    """ExecuteBatch: pools every request into its output.

    Without `status` the call waits for the stream and raises on error; with
    `status` it returns right after the launches and the result is read with
    status.wait().
    """
    if isinstance(requests, PreparedBatch):
      arr, names = requests.array, None
    else:
      arr, names = self._c_requests(requests)
    flags = C.EXEC_FUSED if fused else C.EXEC_STRICT
    if status is not None:
      flags |= C.EXEC_ASYNC
    rc = C.lib.xse_engine_execute_batch(
        self._handle, arr, len(requests), stream_handle(stream), flags,
        status.handle if status is not None else None)
    del names
    C.check(rc)

  def execute_interaction(self, requests: Sequence[BagRequest], dense, out,
                          *, stream=None, fused=False,
                          status: Optional[Status] = None, out_lo=None):
    """Pools request t (feature t of every sample; `output` unused, may be
    None) and writes the dot interaction of [dense_b; pooled_b,0..T-1] into
    out [batch, >= dim + (T+1)T/2] (fp32): one fused kernel where it serves
    the tables' layout, without writing the pooled rows. Flags and status as
    execute_batch. With `out_lo` (same shape and strides as out), out gets
    each value's TF32 part and out_lo the remainder: the split operands of
    the next three-pass TF32 layer."""
    arr, names = self._c_requests(requests)
    flags = C.EXEC_FUSED if fused else C.EXEC_STRICT
    if status is not None:
      flags |= C.EXEC_ASYNC
    if dense.dtype != torch.float32 or out.dtype != torch.float32:
      raise C.XseError(C.INVALID_ARGUMENT, "dense and out must be float32")
    if dense.dim() != 2 or out.dim() != 2 or dense.stride(1) != 1 or \
        out.stride(1) != 1 or out.shape[0] != dense.shape[0]:
      raise C.XseError(C.INVALID_ARGUMENT,
                       "dense [B, dim] and out [B, width] need unit column "
                       "stride and one batch")
    if out_lo is not None and (out_lo.dtype != torch.float32 or
                               out_lo.shape != out.shape or
                               out_lo.stride() != out.stride()):
      raise C.XseError(C.INVALID_ARGUMENT,
                       "out_lo must match out's shape, strides and dtype")
    rc = C.lib.xse_engine_execute_interaction_tf32(
        self._handle, arr, len(requests), dense.data_ptr(), dense.stride(0),
        dense.shape[0], out.data_ptr(),
        None if out_lo is None else out_lo.data_ptr(), out.stride(0),
        stream_handle(stream), flags,
        status.handle if status is not None else None)
    del names
    C.check(rc)

  def execute_legacy(self, requests: Sequence[BagRequest], *, stream=None):
    """CpuEmbeddingEngine::Execute: per request, a [num_bags, dim] pooled
    array, or [num_bags, max_sequence_length, dim] for a sequence feature,
    in the table's type (float32 or bfloat16; a bf16 table accumulates in
    bf16). The requests' `output` fields are ignored; new tensors are
    returned."""
    outs = []
    for r in requests:
      try:
        table, seq = self.feature_table(r.feature_name)
        info = self.table_info(table)
      except C.XseError:
        outs.append(None)  # the engine call below reports the reference's error
        continue
      dtype = torch.bfloat16 if info.dtype == C.DT_BF16 else torch.float32
      bags = max(r.offsets.numel() - 1, 0)
      shape = (bags, seq, info.dim) if seq > 0 else (bags, info.dim)
      outs.append(torch.empty(shape, dtype=dtype, device=r.offsets.device))
    arr, names = self._c_requests(
        [dataclasses.replace(r, output=o) for r, o in zip(requests, outs)])
    rc = C.lib.xse_engine_execute_legacy(self._handle, arr, len(requests),
                                         stream_handle(stream))
    del names
    C.check(rc)
    return outs

  def set_profiling(self, enable, period=1):
    """Records CUDA events around the pooling kernels of every `period`-th
    execution (the first, the period+1-th, ...) while `enable` is true."""
    C.check(C.lib.xse_engine_set_profiling(self._handle,
                                           int(period) if enable else 0))

  def profile_read(self, with_calls=False):
    """(summed pooling-kernel milliseconds, timed executions) since the last
    read; with `with_calls`, also the number of executions, timed or not."""
    ms = ctypes.c_double()
    n = ctypes.c_int64()
    calls = ctypes.c_int64()
    C.check(C.lib.xse_engine_profile_read(self._handle, ctypes.byref(ms),
                                          ctypes.byref(n),
                                          ctypes.byref(calls)))
    if with_calls:
      return ms.value, n.value, calls.value
    return ms.value, n.value

  def profile_read_stages(self):
    """Since the last read: {"pool_ms", "executions", "validate_ms",
    "validated", "calls"} -- summed pooling and validation kernel times (each
    kernel timed alone, events between them), the timed executions and those
    of them that ran validation kernels, and all executions."""
    ms, vms = ctypes.c_double(), ctypes.c_double()
    n, vn, calls = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    C.check(C.lib.xse_engine_profile_read_stages(
        self._handle, ctypes.byref(vms), ctypes.byref(vn), ctypes.byref(ms),
        ctypes.byref(n), ctypes.byref(calls)))
    return {"pool_ms": ms.value, "executions": n.value,
            "validate_ms": vms.value, "validated": vn.value,
            "calls": calls.value}

  def pool(self, feature_name, ids, offsets, weights=None, *, stream=None,
           fused=False):
    """Single-feature convenience: returns a new [num_bags, dim] tensor."""
    table, _ = self.feature_table(feature_name)
    dim = self.table_info(table).dim
    out = torch.empty((max(offsets.numel() - 1, 0), dim), dtype=torch.float32,
                      device=ids.device if ids is not None else "cuda")
    self.execute_batch([BagRequest(feature_name, ids, offsets, out, weights)],
                       stream=stream, fused=fused)
    return out


def last_launch_count():
  """Kernels launched by this thread's last execute_batch."""
  return C.lib.xse_last_launch_count()


def dot_interaction(dense, pooled, out=None, *, stream=None):
  """DLRM dot interaction: [B, D] dense + [B, T, D] pooled -> [B, D + P]."""
  b, t, d = pooled.shape
  rows = t + 1
  width = d + rows * (rows - 1) // 2
  if out is None:
    out = torch.empty((b, width), dtype=torch.float32, device=pooled.device)
  C.check(C.lib.xse_dot_interaction(
      _ptr(dense.contiguous()), _ptr(pooled.contiguous()), b, t, d, _ptr(out),
      stream_handle(stream)))
  return out
