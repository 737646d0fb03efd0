"""ctypes loader of the CPU oracle (oracle/xse_oracle.cc).

TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke check and by the
benchmark's CPU-baseline leg, never by the product. See xse_oracle.h for what
the oracle restates and how it is pinned.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libxse_oracle.so")

OK, INVALID_ARGUMENT, NOT_FOUND, FAILED_PRECONDITION = 0, 3, 5, 9
F32, BF16, I8_ROWWISE = 0, 1, 2
SUM, MEAN, SQRTN = 1, 2, 3
COMBINE = {"SUM": SUM, "MEAN": MEAN, "SQRT_N": SQRTN, "SQRTN": SQRTN}


class Request(ctypes.Structure):
  _fields_ = [
      ("dtype", ctypes.c_int32),
      ("combine", ctypes.c_int32),
      ("table", ctypes.c_void_p),
      ("scale", ctypes.c_void_p),
      ("bias", ctypes.c_void_p),
      ("vocab", ctypes.c_int64),
      ("dim", ctypes.c_int64),
      ("ids", ctypes.c_void_p),
      ("num_ids", ctypes.c_int64),
      ("offsets", ctypes.c_void_p),
      ("offsets_i64", ctypes.c_int32),
      ("num_offsets", ctypes.c_int64),
      ("weights", ctypes.c_void_p),
      ("num_weights", ctypes.c_int64),
      ("out", ctypes.c_void_p),
  ]


def build():
  subprocess.run(["make", "-s", "-C", HERE], check=True)


def _load():
  if not os.path.exists(LIB_PATH):
    build()
  lib = ctypes.CDLL(LIB_PATH)
  P, I32, I64, U64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64
  lib.oracle_embedding_bag_batch.argtypes = [ctypes.POINTER(Request), I32, I32,
                                             I64, ctypes.c_char_p, I32]
  lib.oracle_assemble_bf16_accumulate.argtypes = [P, I64, I64, I32, P, I64, P,
                                                  I64, P, P, ctypes.c_char_p,
                                                  I32]
  lib.oracle_sequence_gather.argtypes = [P, I32, I64, I64, P, P, I64, I64, P,
                                         P, I32]
  lib.oracle_dense_to_csr.argtypes = [P, I32, I64, I64, I64, P, P, P,
                                      ctypes.c_char_p, I32]
  lib.oracle_dense_lookup_row_pointers.argtypes = [I64, I64, P,
                                                   ctypes.c_char_p, I32]
  lib.oracle_dot_interaction.argtypes = [P, P, I64, I32, I32, P]
  lib.oracle_dot_interaction.restype = None
  lib.oracle_uniform.argtypes = [U64, U64, U64]
  lib.oracle_uniform.restype = ctypes.c_double
  lib.oracle_synth_rows_f32.argtypes = [U64, U64, I64, I64, I64, P]
  lib.oracle_synth_rows_f32.restype = None
  lib.oracle_synth_rows_bf16.argtypes = [U64, U64, I64, I64, I64, P]
  lib.oracle_synth_rows_bf16.restype = None
  lib.oracle_synth_rows_i8.argtypes = [U64, U64, I64, I64, I64, P, P, P]
  lib.oracle_synth_rows_i8.restype = None
  lib.oracle_synth_rows_at.argtypes = [I32, U64, U64, P, I64, I64, P, P, P]
  lib.oracle_synth_rows_at.restype = None
  lib.oracle_synth_lengths.argtypes = [I64, I32, I32, U64, U64, P]
  lib.oracle_synth_lengths.restype = None
  lib.oracle_synth_weights.argtypes = [I64, U64, U64, I64, P]
  lib.oracle_synth_weights.restype = None
  lib.oracle_synth_ids.argtypes = [I64, I64, ctypes.c_double, U64, U64, U64,
                                   U64, I64, P]
  lib.oracle_synth_ids.restype = None
  lib.oracle_zipf_rank.argtypes = [U64, U64, U64, I64, ctypes.c_double]
  lib.oracle_zipf_rank.restype = I64
  lib.oracle_host_cores.argtypes = []
  lib.oracle_host_cores.restype = I32
  return lib


lib = _load()


class OracleError(RuntimeError):

  def __init__(self, code, message):
    super().__init__(f"{code}: {message}")
    self.code = code
    self.message = message


def _p(a):
  return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def host_cores():
  return lib.oracle_host_cores()


class Bag:
  """One request for the oracle, on numpy arrays."""

  def __init__(self, table, ids, offsets, weights=None, combine="SUM",
               dtype=F32, scale=None, bias=None, out=None):
    self.table = np.ascontiguousarray(table)
    self.ids = np.ascontiguousarray(ids, dtype=np.int64)
    self.offsets = np.ascontiguousarray(offsets)
    assert self.offsets.dtype in (np.int32, np.int64)
    self.weights = None if weights is None else np.ascontiguousarray(
        weights, dtype=np.float32)
    self.combine = COMBINE[combine] if isinstance(combine, str) else combine
    self.dtype = dtype
    self.scale = None if scale is None else np.ascontiguousarray(
        scale, dtype=np.float32)
    self.bias = None if bias is None else np.ascontiguousarray(
        bias, dtype=np.float32)
    dim = self.table.shape[1]
    self.out = out if out is not None else np.zeros(
        (max(len(self.offsets) - 1, 0), dim), dtype=np.float32)

  def c_request(self):
    return Request(
        dtype=self.dtype, combine=self.combine, table=_p(self.table),
        scale=_p(self.scale), bias=_p(self.bias), vocab=self.table.shape[0],
        dim=self.table.shape[1], ids=_p(self.ids), num_ids=len(self.ids),
        offsets=_p(self.offsets),
        offsets_i64=1 if self.offsets.dtype == np.int64 else 0,
        num_offsets=len(self.offsets), weights=_p(self.weights),
        num_weights=0 if self.weights is None else len(self.weights),
        out=_p(self.out))


def embedding_bag_batch(bags, num_threads=1, inline_threshold=65536):
  """ExecuteEmbeddingBagBatch restatement; raises OracleError on failure."""
  arr = (Request * len(bags))(*[b.c_request() for b in bags])
  err = ctypes.create_string_buffer(1024)
  rc = lib.oracle_embedding_bag_batch(arr, len(bags), num_threads,
                                      inline_threshold, err, len(err))
  if rc != OK:
    raise OracleError(rc, err.value.decode())
  return [b.out for b in bags]


def embedding_bag(table, ids, offsets, weights=None, combine="SUM", dtype=F32,
                  scale=None, bias=None, num_threads=1):
  bag = Bag(table, ids, offsets, weights, combine, dtype, scale, bias)
  return embedding_bag_batch([bag], num_threads)[0]


def assemble_bf16_accumulate(table_bits, ids, row_pointers, weights=None,
                             combine="SUM"):
  """Reference bf16 path (bf16 accumulator); returns bf16 bits as uint16."""
  table_bits = np.ascontiguousarray(table_bits, dtype=np.uint16)
  ids = np.ascontiguousarray(ids, dtype=np.int64)
  rp = np.ascontiguousarray(row_pointers, dtype=np.int32)
  w = None if weights is None else np.ascontiguousarray(weights, np.float32)
  out = np.zeros((len(rp) - 1, table_bits.shape[1]), dtype=np.uint16)
  err = ctypes.create_string_buffer(1024)
  rc = lib.oracle_assemble_bf16_accumulate(
      _p(table_bits), table_bits.shape[0], table_bits.shape[1],
      COMBINE[combine], _p(ids), len(ids), _p(rp), len(rp), _p(w), _p(out),
      err, len(err))
  if rc != OK:
    raise OracleError(rc, err.value.decode())
  return out


def sequence_gather(table, ids, row_pointers, max_seq, dtype=F32):
  """AssembleSequenceEmbeddings restatement: [samples, max_seq, dim] of the
  table's type (fp32, or bf16 bits as uint16)."""
  table = np.ascontiguousarray(table)
  ids = np.ascontiguousarray(ids, dtype=np.int64)
  rp = np.ascontiguousarray(row_pointers, dtype=np.int32)
  out = np.zeros((len(rp) - 1, max_seq, table.shape[1]), dtype=table.dtype)
  err = ctypes.create_string_buffer(1024)
  rc = lib.oracle_sequence_gather(_p(table), dtype, table.shape[0],
                                  table.shape[1], _p(ids), _p(rp), len(rp),
                                  max_seq, _p(out), err, len(err))
  if rc != OK:
    raise OracleError(rc, err.value.decode())
  return out


def dense_to_csr(dense, pad_value=0):
  dense = np.ascontiguousarray(dense)
  assert dense.dtype in (np.int32, np.int64)
  batch = dense.shape[0]
  seq = dense.size // batch if batch > 0 else 0
  ids = np.zeros(batch * seq + batch, dtype=np.int64)
  rp = np.zeros(batch + 1, dtype=np.int32)
  n = ctypes.c_int64()
  err = ctypes.create_string_buffer(1024)
  rc = lib.oracle_dense_to_csr(_p(dense), 1 if dense.dtype == np.int64 else 0,
                               batch, seq, pad_value, _p(ids), _p(rp),
                               ctypes.byref(n), err, len(err))
  if rc != OK:
    raise OracleError(rc, err.value.decode())
  return ids[:n.value], rp


def dense_lookup_row_pointers(batch, valency, materialize=True):
  rp = np.zeros(batch + 1, dtype=np.int32) if materialize else None
  err = ctypes.create_string_buffer(1024)
  rc = lib.oracle_dense_lookup_row_pointers(batch, valency, _p(rp), err,
                                            len(err))
  if rc != OK:
    raise OracleError(rc, err.value.decode())
  return rp


def dot_interaction(dense, pooled):
  dense = np.ascontiguousarray(dense, dtype=np.float32)
  pooled = np.ascontiguousarray(pooled, dtype=np.float32)
  b, t, d = pooled.shape
  rows = t + 1
  out = np.zeros((b, d + rows * (rows - 1) // 2), dtype=np.float32)
  lib.oracle_dot_interaction(_p(dense), _p(pooled), b, t, d, _p(out))
  return out


def synth_rows(dtype, seed, table, row0, nrows, dim):
  if dtype == F32:
    out = np.zeros((nrows, dim), dtype=np.float32)
    lib.oracle_synth_rows_f32(seed, table, row0, nrows, dim, _p(out))
    return out, None, None
  if dtype == BF16:
    out = np.zeros((nrows, dim), dtype=np.uint16)
    lib.oracle_synth_rows_bf16(seed, table, row0, nrows, dim, _p(out))
    return out, None, None
  q = np.zeros((nrows, dim), dtype=np.int8)
  s = np.zeros(nrows, dtype=np.float32)
  b = np.zeros(nrows, dtype=np.float32)
  lib.oracle_synth_rows_i8(seed, table, row0, nrows, dim, _p(q), _p(s), _p(b))
  return q, s, b


def zipf_rank(seed, stream, index, n, alpha):
  return lib.oracle_zipf_rank(seed, stream, index, n, alpha)


def bf16_bits_to_f32(bits):
  return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(
      np.float32)


def synth_rows_at(dtype, seed, table, rows, dim):
  """Rows `rows` (any order) of a synthetic table: (values, scale, bias) as
  synth_rows returns them."""
  rows = np.ascontiguousarray(rows, dtype=np.int64)
  n = len(rows)
  vdt = {F32: np.float32, BF16: np.uint16, I8_ROWWISE: np.int8}[dtype]
  out = np.zeros((n, dim), dtype=vdt)
  scale = bias = None
  if dtype == I8_ROWWISE:
    scale = np.zeros(n, dtype=np.float32)
    bias = np.zeros(n, dtype=np.float32)
  lib.oracle_synth_rows_at(dtype, seed, table, _p(rows), n, dim, _p(out),
                           _p(scale), _p(bias))
  return out, scale, bias


def synth_lengths(n, lo, hi, seed, table):
  out = np.zeros(n, dtype=np.int64)
  lib.oracle_synth_lengths(n, lo, hi, seed, table, _p(out))
  return out


def synth_weights(n, seed, table, index0=0):
  out = np.zeros(n, dtype=np.float32)
  lib.oracle_synth_weights(n, seed, table, index0, _p(out))
  return out


def synth_ids(n, vocab, seed, table, alpha=0.0, perm_mul=1, perm_add=0,
              index0=0):
  out = np.zeros(n, dtype=np.int64)
  lib.oracle_synth_ids(n, vocab, float(alpha), perm_mul, perm_add, seed,
                       table, index0, _p(out))
  return out


def compare_pooled(got, want, bound=None, rtol=1e-5):
  """Pooled rows against the oracle's: bit for bit when `bound` is None,
  else |got - want| <= rtol * bound per element (the condition-aware bound
  of int8 row-wise tables). Returns a summary dict."""
  got = np.asarray(got, dtype=np.float32)
  want = np.asarray(want, dtype=np.float32)
  same = (got.view(np.uint32) == want.view(np.uint32)) | (
      np.isnan(got) & np.isnan(want))
  err = np.abs(got.astype(np.float64) - want.astype(np.float64))
  scale = np.maximum(np.abs(want.astype(np.float64)), 1e-30)
  out = {"elements": int(got.size), "bit_exact": bool(same.all()),
         "mismatched": int((~same).sum()),
         "max_abs_err": float(err.max()) if err.size else 0.0,
         "max_rel_err": float((err / scale).max()) if err.size else 0.0}
  if bound is None:
    out["ok"] = out["bit_exact"]
    out["rule"] = "bit-exact"
  else:
    lim = rtol * np.asarray(bound, dtype=np.float64)
    out["ok"] = bool((err <= lim).all())
    out["rule"] = f"|err| <= {rtol:g} x sum|w|(|q|s + |b|)"
  return out


def sampled_bags(num_bags, count, seed, lengths=None):
  """Bag indices to check: the first and last bags, the longest (when
  `lengths` is given) and a seeded random sample, sorted, without
  repeats."""
  rng = np.random.default_rng(seed)
  pick = set(rng.choice(num_bags, size=min(count, num_bags), replace=False)
             .tolist())
  pick.update({0, num_bags - 1})
  if lengths is not None and len(lengths):
    pick.add(int(np.argmax(lengths)))
  return np.array(sorted(pick), dtype=np.int64)


def pool_sampled(dtype, seed, table, dim, combine, ids, offsets, weights,
                 bags, window=None, num_threads=4):
  """The oracle's pooled rows for bags `bags` of one request (ids, offsets
  and weights as numpy arrays over the whole batch, offsets absolute),
  with the touched rows regenerated from the counter RNG instead of
  materialising the table. `window` (row_begin, row_end): a row-wise shard;
  ids outside it contribute nothing, while bag lengths and weight sums count
  every id. Returns (rows [len(bags), dim], bound or None)."""
  offsets = np.asarray(offsets, dtype=np.int64)
  starts, ends = offsets[bags], offsets[bags + 1]
  pos = np.concatenate([np.arange(a, b, dtype=np.int64)
                        for a, b in zip(starts, ends)] or
                       [np.zeros(0, np.int64)])
  sub_ids = np.asarray(ids, dtype=np.int64)[pos]
  sub_w = None if weights is None else np.asarray(weights, np.float32)[pos]
  sub_off = np.concatenate([[0], np.cumsum(ends - starts)]).astype(np.int64)
  uniq, local = np.unique(sub_ids, return_inverse=True)
  vals, scale, bias = synth_rows_at(dtype, seed, table, uniq, dim)
  if window is not None:
    outside = (uniq < window[0]) | (uniq >= window[1])
    vals[outside] = 0
    if scale is not None:
      scale[outside] = 0.0
      bias[outside] = 0.0
  want = embedding_bag(vals, local, sub_off, sub_w, combine, dtype, scale,
                       bias, num_threads=num_threads)
  bound = None
  if dtype == I8_ROWWISE:
    bound = embedding_bag(np.abs(vals.astype(np.int16)).astype(np.int8),
                          local, sub_off,
                          None if sub_w is None else np.abs(sub_w), combine,
                          dtype, np.abs(scale), np.abs(bias),
                          num_threads=num_threads)
  return want, bound
