"""GPU test of the allocation-free pooling entry point.

xse_engine_execute_batch_noalloc serves callers that may not allocate GPU
memory while handling a request -- a plugin whose host framework owns every
device buffer, or a latency-critical serving thread where cudaMalloc would
synchronize the device. Instead of an allocated status block it keeps its
validation status in one fixed device array. This test calls it through the
C ABI and checks that two calls in a row produce exactly what the regular
xse_engine_execute_batch produces (bit for bit) and what the oracle produces
(bit for bit for fp32 and bf16 tables, within the int8 tolerance of the other
pooling tests for int8 tables), that an error leaves no stale status for the
next call, that groups mixing errors in several requests report the same
error as the regular call, and that groups beyond the array's capacity are
rejected.

The file name makes pytest collect it last; it also runs on its own.
"""

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import (assert_bitwise, assert_pooled, expect_pool,
                            random_csr, random_table, to_dev)

pytestmark = pytest.mark.gpu

TABLES = [  # (name, dtype, dim, combine, weighted)
    ("bf16_wsum", oracle.BF16, 128, "SUM", True),
    ("f32_mean", oracle.F32, 64, "MEAN", False),
    ("i8_sqrtn", oracle.I8_ROWWISE, 32, "SQRT_N", True),
]


def build(xse, rng):
  eng = xse.EmbeddingEngine(0)
  inputs, expected = [], []
  for k, (name, dtype, dim, combine, weighted) in enumerate(TABLES):
    vocab = 700 + 13 * k
    host, dev, scale, bias = random_table(rng, dtype, vocab, dim)
    eng.add_table(name, dev, combine, scale=scale, bias=bias)
    eng.register_feature(name, name)
    ids, offsets = random_csr(rng, vocab, 150 + k, 45, first=3 * k)
    w = rng.uniform(0, 1, len(ids)).astype(np.float32) if weighted else None
    offsets = offsets.astype(np.int32 if k == 1 else np.int64)
    inputs.append((name, dim, to_dev(ids), to_dev(offsets),
                   None if w is None else to_dev(w)))
    expected.append(expect_pool(host, dtype, ids, offsets, w, combine, scale,
                                bias))
  return eng, inputs, expected


def requests(xse, inputs):
  outs, reqs = [], []
  for name, dim, ids, offsets, w in inputs:
    out = torch.full((offsets.numel() - 1, dim), -7.0, device="cuda")
    outs.append(out)
    reqs.append(xse.BagRequest(name, ids, offsets, out, w))
  return outs, reqs


def call_noalloc(xse, eng, arr, n):
  rc = xse._capi.lib.xse_engine_execute_batch_noalloc(
      eng.handle, arr, n, xse.stream_handle())
  return rc, xse._capi.last_error()


def call_regular(xse, eng, arr, n):
  rc = xse._capi.lib.xse_engine_execute_batch(
      eng.handle, arr, n, xse.stream_handle(), xse._capi.EXEC_STRICT, None)
  return rc, xse._capi.last_error()


def noalloc(xse, eng, reqs):
  arr, names = eng._c_requests(reqs)
  result = call_noalloc(xse, eng, arr, len(reqs))
  del names
  return result


def test_noalloc_matches_regular_entry_point_and_oracle(xse):
  rng = np.random.default_rng(2026)
  eng, inputs, expected = build(xse, rng)
  want, reqs = requests(xse, inputs)
  eng.execute_batch(reqs)
  for call in range(2):  # two calls in a row share the fixed scratch array
    got, reqs = requests(xse, inputs)
    rc, msg = noalloc(xse, eng, reqs)
    assert rc == xse._capi.OK, msg
    for k, (g, w, e) in enumerate(zip(got, want, expected)):
      g = g.cpu().numpy()
      assert_bitwise(g, w.cpu().numpy(), f"noalloc call {call} table {k}")
      assert_pooled(g, e, f"noalloc call {call} table {k} vs oracle")
  eng.close()


def test_noalloc_errors_and_limits(xse):
  rng = np.random.default_rng(7)
  eng, inputs, _ = build(xse, rng)
  name, dim, ids, offsets, w = inputs[1]
  bad = ids.clone()
  bad[5] = 10_000
  out = torch.zeros((offsets.numel() - 1, dim), device="cuda")
  bad_req = [xse.BagRequest(name, bad, offsets, out, w)]
  with pytest.raises(xse.XseError) as regular:
    eng.execute_batch(bad_req)
  rc, msg = noalloc(xse, eng, bad_req)
  assert rc == regular.value.code and msg == regular.value.message
  # The failed call's status must not leak into the next one.
  got, reqs = requests(xse, inputs)
  rc, msg = noalloc(xse, eng, reqs)
  assert rc == xse._capi.OK, msg
  want, reqs = requests(xse, inputs)
  eng.execute_batch(reqs)
  for g, wv in zip(got, want):
    assert_bitwise(g.cpu().numpy(), wv.cpu().numpy(), "after error")
  # Groups beyond the fixed array are rejected before any launch.
  limit = 64
  many = [xse.BagRequest(name, ids, offsets,
                         torch.empty((offsets.numel() - 1, dim), device="cuda"),
                         w) for _ in range(limit + 1)]
  rc, msg = noalloc(xse, eng, many)
  assert rc == xse._capi.INVALID_ARGUMENT
  assert "at most 64 requests" in msg
  eng.close()


def mixed_cases(xse, eng, inputs):
  """Groups whose requests fail in different ways, as (label, ctypes request
  array, keep-alive list). Each is built from fresh outputs."""
  C = xse._capi
  cases = []

  # (a) request 0: an out-of-range id; request 1: null weights.
  outs, reqs = requests(xse, inputs)
  bad = inputs[0][2].clone()
  bad[7] = -3
  reqs[0].ids = bad
  arr, names = eng._c_requests(reqs)
  arr[1].weights = None
  arr[1].num_weights = 5
  cases.append(("bad id, then null weights", arr, [names, outs, reqs, bad]))

  # (b) request 0: decreasing offsets; request 1: its output overlaps
  # request 0's ids.
  outs, reqs = requests(xse, inputs)
  offs = inputs[0][3].clone()
  a, b = int(offs[3]), int(offs[4])
  offs[3] = b + 1
  offs[4] = a
  reqs[0].offsets = offs
  ids0 = inputs[0][2]
  arr, names = eng._c_requests(reqs)
  arr[1].output = ids0.data_ptr()
  cases.append(("bad offsets, then output over ids", arr,
                [names, outs, reqs, offs]))

  # (c) request 0: an out-of-range id; request 1: an unknown index type.
  outs, reqs = requests(xse, inputs)
  bad = inputs[0][2].clone()
  bad[9] = 1 << 40
  reqs[0].ids = bad
  arr, names = eng._c_requests(reqs)
  arr[1].ids_type = 7
  cases.append(("bad id, then bad index type", arr, [names, outs, reqs, bad]))

  # (d) request 0 valid; request 1: null ids; request 2: bad offsets.
  outs, reqs = requests(xse, inputs)
  offs = inputs[2][3].clone()
  offs[0] = -1
  reqs[2].offsets = offs
  arr, names = eng._c_requests(reqs)
  arr[1].ids = None
  cases.append(("null ids, then bad offsets", arr, [names, outs, reqs, offs]))

  # (e) every request valid on its own; two outputs overlap inputs, and
  # request 2's output sits at a lower address than request 0's, so the
  # address-ordered scan names request 2 first (a scan in request order
  # would name request 0). The inputs are copied into the shared buffer, so
  # every id, offset and weight is still valid.
  outs, reqs = requests(xse, inputs)
  pool = torch.zeros(1 << 16, device="cuda")
  ids0, w2 = inputs[0][2], inputs[2][4]
  pool[16:16 + w2.numel()] = w2
  pool[20064:20064 + 2 * ids0.numel()].view(torch.int64).copy_(ids0)
  arr, names = eng._c_requests(reqs)
  arr[2].output = pool.data_ptr()
  arr[2].weights = pool.data_ptr() + 4 * 16
  arr[0].output = pool.data_ptr() + 4 * 20000
  arr[0].ids = pool.data_ptr() + 4 * 20064
  assert arr[0].ids_type == C.INDEX_I64
  cases.append(("two outputs over inputs", arr, [names, outs, reqs, pool]))

  # (f) outputs of requests 1 and 2 overlap each other.
  outs, reqs = requests(xse, inputs)
  arr, names = eng._c_requests(reqs)
  arr[2].output = arr[1].output
  cases.append(("overlapping outputs", arr, [names, outs, reqs]))
  return cases


def test_noalloc_reports_errors_in_the_regular_order(xse):
  rng = np.random.default_rng(99)
  eng, inputs, _ = build(xse, rng)
  for label, arr, keep in mixed_cases(xse, eng, inputs):
    want = call_regular(xse, eng, arr, len(arr))
    got = call_noalloc(xse, eng, arr, len(arr))
    assert want[0] != xse._capi.OK, label
    assert got == want, (label, got, want)
    del keep
  # A valid group still pools correctly afterwards.
  got, reqs = requests(xse, inputs)
  rc, msg = noalloc(xse, eng, reqs)
  assert rc == xse._capi.OK, msg
  want, reqs = requests(xse, inputs)
  eng.execute_batch(reqs)
  for g, w in zip(got, want):
    assert_bitwise(g.cpu().numpy(), w.cpu().numpy(), "after mixed errors")
  eng.close()
