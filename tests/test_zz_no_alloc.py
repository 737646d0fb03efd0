"""GPU test of the allocation-free pooling entry point.

xse_engine_execute_batch_noalloc serves callers that may not allocate GPU
memory while handling a request -- a plugin whose host framework owns every
device buffer, or a latency-critical serving thread where cudaMalloc would
synchronize the device. Instead of an allocated status block it keeps its
validation status in one fixed device array. This test calls it through the
C ABI and checks that two calls in a row produce exactly what the regular
xse_engine_execute_batch produces (bit for bit, the tolerance of the other
pooling tests), that an error leaves no stale status for the next call, and
that groups beyond the array's capacity are rejected.

The file name makes pytest collect it last; it also runs on its own.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import assert_bitwise, random_csr, random_table, to_dev

pytestmark = pytest.mark.gpu

TABLES = [  # (name, dtype, dim, combine, weighted)
    ("bf16_wsum", oracle.BF16, 128, "SUM", True),
    ("f32_mean", oracle.F32, 64, "MEAN", False),
    ("i8_sqrtn", oracle.I8_ROWWISE, 32, "SQRT_N", True),
]


def build(xse, rng):
  eng = xse.EmbeddingEngine(0)
  inputs = []
  for k, (name, dtype, dim, combine, weighted) in enumerate(TABLES):
    vocab = 700 + 13 * k
    _, dev, scale, bias = random_table(rng, dtype, vocab, dim)
    eng.add_table(name, dev, combine, scale=scale, bias=bias)
    eng.register_feature(name, name)
    ids, offsets = random_csr(rng, vocab, 150 + k, 45, first=3 * k)
    w = rng.uniform(0, 1, len(ids)).astype(np.float32) if weighted else None
    inputs.append((name, dim, to_dev(ids),
                   to_dev(offsets.astype(np.int32 if k == 1 else np.int64)),
                   None if w is None else to_dev(w)))
  return eng, inputs


def requests(xse, inputs):
  outs, reqs = [], []
  for name, dim, ids, offsets, w in inputs:
    out = torch.full((offsets.numel() - 1, dim), -7.0, device="cuda")
    outs.append(out)
    reqs.append(xse.BagRequest(name, ids, offsets, out, w))
  return outs, reqs


def call_noalloc(xse, eng, reqs):
  arr, names = eng._c_requests(reqs)
  rc = xse._capi.lib.xse_engine_execute_batch_noalloc(
      eng.handle, arr, len(reqs), xse.stream_handle())
  del names
  return rc, xse._capi.last_error()


def test_noalloc_matches_regular_entry_point(xse):
  rng = np.random.default_rng(2026)
  eng, inputs = build(xse, rng)
  want, reqs = requests(xse, inputs)
  eng.execute_batch(reqs)
  for _ in range(2):  # two calls in a row share the fixed scratch array
    got, reqs = requests(xse, inputs)
    rc, msg = call_noalloc(xse, eng, reqs)
    assert rc == xse._capi.OK, msg
    for g, w in zip(got, want):
      assert_bitwise(g.cpu().numpy(), w.cpu().numpy(), "noalloc")
  eng.close()


def test_noalloc_errors_and_limits(xse):
  rng = np.random.default_rng(7)
  eng, inputs = build(xse, rng)
  name, dim, ids, offsets, w = inputs[1]
  bad = ids.clone()
  bad[5] = 10_000
  out = torch.zeros((offsets.numel() - 1, dim), device="cuda")
  bad_req = [xse.BagRequest(name, bad, offsets, out, w)]
  with pytest.raises(xse.XseError) as regular:
    eng.execute_batch(bad_req)
  rc, msg = call_noalloc(xse, eng, bad_req)
  assert rc == regular.value.code and msg == regular.value.message
  # The failed call's status must not leak into the next one.
  got, reqs = requests(xse, inputs)
  rc, msg = call_noalloc(xse, eng, reqs)
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
  rc, msg = call_noalloc(xse, eng, many)
  assert rc == xse._capi.INVALID_ARGUMENT
  assert "at most 64 requests" in msg
  assert ctypes.sizeof(xse._capi.BagRequest) > 0
  eng.close()
