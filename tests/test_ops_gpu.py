"""GPU tests of the operator layer through its C ABI (include/xse_ops.h),
written after the reference's own operator and resource tests:
data/kernels/cpu_embedding/cpu_embedding_lookup_transform_test.cc,
dense_cpu_embedding_lookup_transform_test.cc, cpu_embedding_resource_test.cc
and data/ops/cpu_embedding_test.py. Known answers are compared exactly and
against the oracle bit for bit; error messages exactly."""

import os

import numpy as np
import pytest

from oracle import oracle
from parity_helpers import assert_pooled, expect_pool

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(xse):
  from xla_serving_b200 import ops as ops_module  # pylint: disable=import-outside-toplevel
  return ops_module


def make_resource(ops, tables, dims=None):
  """An empty resource filled like TestCpuEmbeddingEngineResource
  (cpu_embedding_lookup_transform_test.cc:58-66)."""
  res = ops.CpuEmbeddingResource.empty()
  eng = res.engine
  for name, (data, combine) in tables.items():
    eng.add_table(name, np.asarray(data, np.float32), combine)
    eng.register_feature(name.replace("table", "feature"), name)
  for feature, dim in (dims or {}).items():
    res.register_embedding_dim(feature, dim)
  return res


TABLE1 = {"table1": ([[1, 2, 3], [4, 5, 6]], "SUM")}


def test_execute_weighted_sum(ops):
  # cpu_embedding_lookup_transform_test.cc:93-167
  res = make_resource(ops, TABLE1, {"feature1": 3})
  t = ops.CpuEmbeddingLookupTransform(res, ["feature1"])
  out, = t([np.array([0, 0, 1], np.int64)], [np.array([0, 1, 3], np.int32)],
           [np.array([1.0, 0.5, 0.5], np.float32)])
  assert out.shape == (2, 3)
  np.testing.assert_array_equal(out.ravel(), [1, 2, 3, 2.5, 3.5, 4.5])


def test_dense_execute(ops):
  # cpu_embedding_lookup_transform_test.cc:169-233
  res = make_resource(ops, TABLE1, {"feature1": 3})
  t = ops.CpuEmbeddingLookupTransform(res, ["feature1"], dense_lookup=True)
  out, = t([np.array([[0, 1], [1, 0]], np.int32)])
  assert out.shape == (2, 3)
  np.testing.assert_array_equal(out.ravel(), [5, 7, 9, 5, 7, 9])


def test_multi_lookup_mean(ops):
  # cpu_embedding_lookup_transform_test.cc:236-367
  res = make_resource(ops, {
      "tableA": ([[1, 2, 3], [4, 5, 6]], "MEAN"),
      "tableB": ([[7, 8], [9, 10]], "MEAN"),
  })
  eng = res.engine
  eng.register_feature("tableA", "tableA")
  eng.register_feature("tableB", "tableB")
  t = ops.CpuEmbeddingLookupTransform(res, ["tableA", "tableB"])
  a, b = t([np.array([0, 0, 1], np.int64), np.array([1, 1], np.int64)],
           [np.array([0, 1, 3], np.int32), np.array([0, 2], np.int32)],
           [np.array([1, .5, .5], np.float32), np.array([.5, .5], np.float32)])
  assert a.shape == (2, 3) and b.shape == (1, 2)
  np.testing.assert_array_equal(a.ravel(), [1, 2, 3, 2.5, 3.5, 4.5])
  np.testing.assert_array_equal(b.ravel(), [9, 10])


@pytest.mark.parametrize("names,outputs", [
    (["feature1", "feature1"], None),          # DuplicateFeaturesFails
    (["feature1", "feature2"], ["out1", "out1"]),  # DuplicateOutputsFails
    (["feature1", "feature2"], ["out1"]),      # OutputFeatureNamesSizeMismatch
    ([], None),
])
def test_create_rejects(ops, xse, names, outputs):
  # cpu_embedding_lookup_transform_test.cc:425-452
  res = make_resource(ops, TABLE1)
  with pytest.raises(xse.XseError) as e:
    ops.CpuEmbeddingLookupTransform(res, names, output_feature_names=outputs)
  assert e.value.code == xse._capi.INVALID_ARGUMENT


def run_error(ops, xse, ids, rps, weights, dense=False):
  res = make_resource(ops, TABLE1, {"feature1": 3})
  t = ops.CpuEmbeddingLookupTransform(res, ["feature1"], dense_lookup=dense)
  with pytest.raises(xse.XseError) as e:
    t(ids, rps, weights)
  return e.value


def test_lookup_error_messages(ops, xse):
  h = ops.HostBuffer
  i64 = lambda *v: np.array(v, np.int64)  # noqa: E731
  i32 = lambda *v: np.array(v, np.int32)  # noqa: E731
  f32 = lambda *v: np.array(v, np.float32)  # noqa: E731
  cases = [
      # (ids, rps, weights, message) -- cpu_embedding_lookup_transform_test.cc
      ([i64(0)], [np.array(1, np.int32)], [f32(1)],
       "row_pointers HostBuffer must be at least 1D (got scalar)."),  # :370
      ([h(np.array([0.0], np.float32))], [i32(0, 1)], [f32()],
       "Embedding IDs must be int32 or int64."),  # :715
      ([i32(0, 1)], [i32(0)], [f32()],
       "Row pointers must have at least 2 elements."),  # :755
      ([i32(0, 1)], [i32(1, 2)], [f32()],
       "First element of row pointers must be 0."),  # :807
      ([i32(0, 1)], [i32(0, 3)], [f32()],
       "Embedding ids size (2) does not match last element of row pointers "
       "(3)"),  # :858
      ([i32(0, 1)], [i32(0, 2)], [f32(1, 1, 1)],
       "Weights size (3) does not match expected size (2)"),  # :959
      ([i32(0, 1)], [i32(0, 3, 2)], [f32()],
       "FP32 embedding-bag request 0: Row pointers must be non-negative and "
       "monotonic."),  # :910
      ([i32(-1)], [i32(0, 1)], [f32()],
       "FP32 embedding-bag request 0: Embedding ID (-1) at index 0 is out of "
       "bounds [0, 2)."),  # :1011
      ([i32(2)], [i32(0, 1)], [f32()],
       "FP32 embedding-bag request 0: Embedding ID (2) at index 0 is out of "
       "bounds [0, 2)."),  # :1051
      ([h.empty()], [i32(0, 1)], [f32()],
       "ids HostBuffer is uninitialized or null."),
      ([i64(0)], [i32(0, 1)], [h.empty()],
       "weights HostBuffer is uninitialized."),
      ([i64(0)], [i64(0, 1)], [f32()], "Row pointers must be int32 (kS32)."),
  ]
  for ids, rps, weights, message in cases:
    err = run_error(ops, xse, ids, rps, weights)
    assert err.code == xse._capi.INVALID_ARGUMENT, message
    assert err.message == message


def test_lookup_count_and_dense_errors(ops, xse):
  res = make_resource(ops, TABLE1, {"feature1": 3})
  t = ops.CpuEmbeddingLookupTransform(res, ["feature1"], dense_lookup=True)
  with pytest.raises(xse.XseError) as e:
    t([])
  assert e.value.message == ("CpuEmbeddingLookupTransform expected 1 ids "
                             "buffers, but got 0.")
  # Dense overflow checks run before the data is touched
  # (cpu_embedding_lookup_transform_test.cc:622-681): the reference passes a
  # dummy base pointer with a huge shape.
  fake = 0x100000000
  for shape, message in [
      ((2000000, 2000), "Batch volume (batch_size * valency) exceeds "
                        "INT32_MAX bounds."),
      ((2147483648, 1), "Batch size exceeds INT32_MAX bounds."),
      ((4,), "Dense embedding IDs must be a 2D HostBuffer [batch_size, "
             "valency]."),
  ]:
    with pytest.raises(xse.XseError) as e:
      t([ops.HostBuffer(data_ptr=fake, shape=shape)])
    assert e.value.message == message


def dense_resource(ops, tables):
  res = ops.CpuEmbeddingResource.empty()
  eng = res.engine
  for name, (rows, dim) in tables.items():
    data = np.repeat(np.arange(rows, dtype=np.float32)[:, None], dim, axis=1)
    eng.add_table(name, data, "SUM")
  return res, eng


def test_dense_transform_known_answers(ops):
  # dense_cpu_embedding_lookup_transform_test.cc:62-120, :122-206, :350-394
  res, eng = dense_resource(ops, {"table1": (5, 4)})
  eng.register_feature("feat1", "table1")
  res.register_embedding_dim("feat1", 4)
  t = ops.DenseCpuEmbeddingLookupTransform(res, "feat1", pad_value=0)
  out, = t([np.array([[1, 2, 3, 0], [4, 1, 2, 0]], np.int32)])
  np.testing.assert_array_equal(out, [[6] * 4, [7] * 4])
  out64, = t([np.array([[1, 2, 3, 0], [4, 1, 2, 0]], np.int64)])
  np.testing.assert_array_equal(out64, out)

  res2 = ops.CpuEmbeddingResource.empty()
  e2 = res2.engine
  e2.add_table("table1", np.repeat(np.arange(3, dtype=np.float32)[:, None], 4,
                                   axis=1), "SUM")
  e2.add_table("table2", np.array([[0, 0], [10, 10], [20, 20]], np.float32),
               "SUM")
  e2.register_feature("feat1", "table1")
  e2.register_feature("feat2", "table2")
  res2.register_embedding_dim("feat1", 4)
  res2.register_embedding_dim("feat2", 2)
  t2 = ops.DenseCpuEmbeddingLookupTransform(res2, ["feat1", "feat2"])
  a, b = t2([np.array([[1, 2, 0], [2, 2, 0]], np.int32),
             np.array([[1, 0], [2, 1]], np.int32)])
  np.testing.assert_array_equal(a, [[3] * 4, [4] * 4])
  np.testing.assert_array_equal(b, [[10, 10], [30, 30]])

  res3 = ops.CpuEmbeddingResource.empty()
  res3.engine.add_table("table1", np.array([[0, 0], [1, 1]], np.float32),
                        "SUM")
  res3.engine.register_feature("feat1", "table1")
  res3.register_embedding_dim("feat1", 2)
  t3 = ops.DenseCpuEmbeddingLookupTransform(res3, "feat1", pad_value=0)
  out, = t3([np.array([[0, 0, 0]], np.int32)])  # all padding -> row 0
  np.testing.assert_array_equal(out, [[0, 0]])


def test_dense_transform_errors(ops, xse):
  # dense_cpu_embedding_lookup_transform_test.cc:396-536
  res, eng = dense_resource(ops, {"table1": (3, 2)})
  eng.register_feature("feat1", "table1")
  eng.register_feature("seqf", "table1", max_sequence_length=4)
  res.register_embedding_dim("feat1", 2)
  res.register_embedding_dim("seqf", 2)
  with pytest.raises(xse.XseError):
    ops.DenseCpuEmbeddingLookupTransform(res, [])
  with pytest.raises(xse.XseError):
    ops.DenseCpuEmbeddingLookupTransform(res, [""])
  t = ops.DenseCpuEmbeddingLookupTransform(res, "feat1")
  with pytest.raises(xse.XseError) as e:
    t([np.array(1, np.int32)])
  assert e.value.message == "dense_ids for feature feat1 must have rank >= 1."
  with pytest.raises(xse.XseError) as e:
    t([np.zeros((2, 2), np.float32)])
  assert e.value.code == xse._capi.INVALID_ARGUMENT
  with pytest.raises(xse.XseError) as e:
    t([ops.HostBuffer(data_ptr=0x100000000, shape=(2**31, 1))])
  assert e.value.code == xse._capi.INVALID_ARGUMENT
  with pytest.raises(xse.XseError) as e:
    t([np.array([[1]], np.int32), np.array([[1]], np.int32)])
  assert "expected 1 inputs, got 2" in e.value.message
  ts = ops.DenseCpuEmbeddingLookupTransform(res, "seqf")
  with pytest.raises(xse.XseError) as e:
    ts([np.array([[1, 2]], np.int32)])
  assert e.value.code == xse._capi.UNIMPLEMENTED
  assert "non-sequence" in e.value.message


def test_python_known_answers(ops):
  # data/ops/cpu_embedding_test.py:406-477 (resource built from assets)
  res = ops.CpuEmbeddingResource(
      {"feat1": np.array([[0, 0], [1, 1], [2, 2], [3, 3]], np.float32)},
      {"feat1": "SUM"}, [{"name": "feat1", "table_name": "feat1"}])
  t = ops.DenseCpuEmbeddingLookupTransform(res, "feat1", pad_value=0)
  out, = t(np.array([[1, 2, 0], [3, 0, 0]], np.int32))
  np.testing.assert_array_equal(out, [[3, 3], [3, 3]])
  res2 = ops.CpuEmbeddingResource(
      {"feat1": np.array([[0, 0], [1, 2]], np.float32),
       "feat2": np.array([[0, 0, 0], [3, 4, 5]], np.float32)},
      {"feat1": "SUM", "feat2": "SUM"},
      [{"name": "feat1", "table_name": "feat1"},
       {"name": "feat2", "table_name": "feat2"}])
  assert res2.get_embedding_dim("feat2") == 3
  t2 = ops.DenseCpuEmbeddingLookupTransform(res2, ["feat1", "feat2"])
  a, b = t2([np.array([[1, 0]], np.int32), np.array([[1, 0]], np.int32)])
  np.testing.assert_array_equal(a, [[1, 2]])
  np.testing.assert_array_equal(b, [[3, 4, 5]])
  with pytest.raises(ValueError, match="path traversal"):
    ops.CpuEmbeddingResource({"../bad_table": np.ones((1, 1), np.float32)},
                             {"../bad_table": "MEAN"},
                             [{"name": "x", "table_name": "../bad_table"}])


def test_resource_assets_and_errors(ops, xse, tmp_path):
  # cpu_embedding_resource_test.cc:61-293: load from assets, mismatched and
  # missing assets rejected, a failed load can be retried.
  rng = np.random.default_rng(4)
  f32 = rng.uniform(-1, 1, (50, 8)).astype(np.float32)
  bits = (rng.uniform(-1, 1, (40, 16)).astype(np.float32).view(np.uint32)
          >> 16).astype(np.uint16)
  q = rng.integers(-127, 128, (30, 32)).astype(np.int8)
  sc = rng.uniform(1e-3, 1e-2, 30).astype(np.float32)
  bi = rng.uniform(-.1, .1, 30).astype(np.float32)
  res = ops.CpuEmbeddingResource(
      {"a": f32, "b": bits, "c": (q, sc, bi)},
      {"a": "SQRT_N", "b": "SUM", "c": "MEAN"},
      [{"name": "fa", "table_name": "a"}, {"name": "fb", "table_name": "b"},
       {"name": "fc", "table_name": "c"}])
  t = ops.CpuEmbeddingLookupTransform(res, ["fa", "fb", "fc"])
  ids = [rng.integers(0, n, 37) for n in (50, 40, 30)]
  rp = np.array([0, 5, 5, 20, 37], np.int32)
  w = rng.uniform(0, 1, 37).astype(np.float32)
  outs = t(ids, [rp] * 3, [w, np.zeros(0, np.float32), w])
  want = [
      expect_pool(f32, oracle.F32, ids[0], rp, w, "SQRT_N"),
      expect_pool(bits, oracle.BF16, ids[1], rp, None, "SUM"),
      expect_pool(q, oracle.I8_ROWWISE, ids[2], rp, w, "MEAN", sc, bi),
  ]
  for k, (got, exp) in enumerate(zip(outs, want)):
    assert_pooled(got, exp, f"feature {k}")

  # Asset errors.
  manifest = tmp_path / "manifest.textproto"
  table = tmp_path / "t.bin"
  np.ones((4, 2), np.float32).tofile(table)
  manifest.write_text('tables { name: "t" vocab_size: 4 embedding_dim: 2 '
                      'combine_mode: SUM }\n'
                      'feature_specs { name: "f" table: "t" }\n')
  with pytest.raises(xse.XseError) as e:
    ops.CpuEmbeddingResource.from_assets({"t": str(table)})
  assert e.value.message == "Failed to find manifest asset in JCE Resource."
  with pytest.raises(xse.XseError) as e:
    ops.CpuEmbeddingResource.from_assets({"__jce_manifest__": str(manifest)})
  assert e.value.message == "Failed to find table asset: t"
  np.ones((3, 2), np.float32).tofile(table)  # truncated
  with pytest.raises(xse.XseError) as e:
    ops.CpuEmbeddingResource.from_assets(
        {"__jce_manifest__": str(manifest), "t": str(table)})
  assert e.value.message == ("Table asset size mismatch for t. Expected 32 "
                             "bytes, but got 24")
  np.ones((4, 2), np.float32).tofile(table)  # fixed: the retry succeeds
  ok = ops.CpuEmbeddingResource.from_assets(
      {"__jce_manifest__": str(manifest), "t": str(table)})
  assert ok.get_embedding_dim("f") == 2
  with pytest.raises(xse.XseError) as e:
    ok.get_embedding_dim("nope")
  assert e.value.code == xse._capi.NOT_FOUND
  manifest.write_text('tables { name: "t" vocab_size: 4 embedding_dim: 2 }\n')
  with pytest.raises(xse.XseError) as e:
    ops.CpuEmbeddingResource.from_assets(
        {"__jce_manifest__": str(manifest), "t": str(table)})
  assert e.value.message == "Unspecified combine mode for table: t"
  assert os.path.exists(table)


def test_reference_numpy_lookup_through_transform(ops):
  """The reference's numpy lookup fixture through the dense-lookup transform
  with a resource loaded from assets."""
  g = np.load(os.path.join(os.path.dirname(__file__), "golden",
                           "numpy_lookup.npz"))
  n = int(g["num_tables"])
  tables = {f"t{i}": g[f"table_{i}"] for i in range(n)}
  res = ops.CpuEmbeddingResource(
      tables, {k: "SUM" for k in tables},
      [{"name": f"t{i}", "table_name": f"t{i}"} for i in range(n)])
  t = ops.CpuEmbeddingLookupTransform(res, [f"t{i}" for i in range(n)],
                                      dense_lookup=True)
  outs = t([g[f"ids_{i}"] for i in range(n)])
  for i, got in enumerate(outs):
    dense = g[f"ids_{i}"]
    b, v = dense.shape
    exact = oracle.embedding_bag(g[f"table_{i}"], dense.ravel(),
                                 np.arange(b + 1, dtype=np.int32) * v)
    np.testing.assert_array_equal(got, exact)
    np.testing.assert_allclose(got, g[f"out_{i}"], rtol=1e-5, atol=1e-6)


def test_pinned_and_pageable_inputs(ops):
  """Pinned inputs go to the device directly, pageable ones through the
  staging block; mixed in one call, results match the oracle bit for bit,
  and pinned outputs (copy=False) hold the same values."""
  rng = np.random.default_rng(11)
  vocab, dim, batch = 300, 24, 17
  tables = {f"table{i}": (rng.standard_normal((vocab, dim)).astype(np.float32),
                          mode)
            for i, mode in enumerate(["SUM", "MEAN", "SQRT_N"])}
  res = make_resource(ops, tables)
  names = [f"feature{i}" for i in range(3)]
  t = ops.CpuEmbeddingLookupTransform(res, names)
  ids, rps, ws, pinned = [], [], [], []
  for i in range(3):
    lengths = rng.integers(0, 6, batch)
    rp = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    n = int(rp[-1])
    idv = rng.integers(0, vocab, n).astype(np.int64)
    wv = rng.random(n).astype(np.float32)
    # feature 0: all pinned; feature 1: pinned ids only; feature 2: pageable.
    if i < 2:
      b = ops.PinnedBuffer((n,), np.int64)
      b.array[:] = idv
      pinned.append(b)
      ids.append(b)
    else:
      ids.append(idv)
    if i == 0:
      b = ops.PinnedBuffer((batch + 1,), np.int32)
      b.array[:] = rp
      w = ops.PinnedBuffer((n,), np.float32)
      w.array[:] = wv
      pinned += [b, w]
      rps.append(b)
      ws.append(w)
    else:
      rps.append(rp)
      ws.append(wv)
  want = [oracle.embedding_bag(tables[f"table{i}"][0],
                               ids[i].array if i < 2 else ids[i],
                               rps[i].array if i == 0 else rps[i],
                               ws[i].array if i == 0 else ws[i],
                               tables[f"table{i}"][1])
          for i in range(3)]
  outs = t(ids, rps, ws)
  for got, exp in zip(outs, want):
    np.testing.assert_array_equal(got, exp)
  held = t(ids, rps, ws, copy=False)
  for got, exp in zip(held, want):
    assert isinstance(got, ops.PinnedBuffer)
    np.testing.assert_array_equal(got.array, exp)
    got.close()
  for b in pinned:
    b.close()


def test_concurrent_calls_from_threads(ops):
  """Calls of one transform from several threads on their own streams run
  concurrently (each takes its own staging slot); every call's outputs
  match the oracle bit for bit."""
  import threading  # pylint: disable=import-outside-toplevel
  import torch  # pylint: disable=import-outside-toplevel
  rng = np.random.default_rng(21)
  vocab, dim = 4000, 32
  table = rng.standard_normal((vocab, dim)).astype(np.float32)
  res = make_resource(ops, {"table0": (table, "MEAN")})
  t = ops.CpuEmbeddingLookupTransform(res, ["feature0"])
  cases = []
  for k in range(12):
    lengths = rng.integers(0, 30, 300)
    rp = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    ids = rng.integers(0, vocab, int(rp[-1])).astype(np.int64)
    w = rng.random(len(ids)).astype(np.float32)
    cases.append((ids, rp, w, oracle.embedding_bag(table, ids, rp, w,
                                                   "MEAN")))
  results = [None] * len(cases)
  errors = []

  def worker(start):
    try:
      stream = torch.cuda.Stream()
      for k in range(start, len(cases), 3):
        ids, rp, w, _ = cases[k]
        results[k], = t([ids], [rp], [w], stream=stream)
    except Exception as e:  # pylint: disable=broad-except
      errors.append(e)

  threads = [threading.Thread(target=worker, args=(s,)) for s in range(3)]
  for th in threads:
    th.start()
  for th in threads:
    th.join()
  assert not errors, errors
  for k, case in enumerate(cases):
    np.testing.assert_array_equal(results[k], case[3])


@pytest.mark.parametrize("dtype,batch,seq,pad", [
    (np.int32, 5000, 37, 0), (np.int64, 1200, 300, 7), (np.int32, 3, 1, 5),
    (np.int64, 4097, 2, -1)])
def test_dense_transform_device_csr(ops, dtype, batch, seq, pad):
  """The CSR built on the device (pad filter, all-pad rows keeping one pad
  id, scanned row pointers) pools to the oracle's CSR + pooling bit for
  bit, across multi-block scans, both id types and odd shapes."""
  rng = np.random.default_rng(batch + seq)
  vocab, dim = 997, 24
  table = rng.standard_normal((vocab, dim)).astype(np.float32)
  res = ops.CpuEmbeddingResource.empty()
  res.engine.add_table("t", table, "MEAN")
  res.engine.register_feature("f", "t")
  res.register_embedding_dim("f", dim)
  t = ops.DenseCpuEmbeddingLookupTransform(res, "f", pad_value=pad)
  dense = rng.integers(0, vocab, (batch, seq)).astype(dtype)
  dense[rng.random((batch, seq)) < 0.4] = pad
  dense[rng.random(batch) < 0.05] = pad  # some all-pad rows
  if pad < 0:
    dense[dense == pad] = 3  # an out-of-range pad must never be kept
  got, = t([dense])
  ids, rp = oracle.dense_to_csr(dense, pad)
  want = oracle.embedding_bag(table, ids, rp, None, "MEAN")
  np.testing.assert_array_equal(got, want)


def test_dense_transform_bad_id_message_from_device_csr(ops, xse):
  """An out-of-range id is reported at its position in the CSR (after the
  pad filter), exactly as when the CSR is built on the host."""
  res = ops.CpuEmbeddingResource.empty()
  res.engine.add_table("t", np.ones((10, 4), np.float32), "SUM")
  res.engine.register_feature("f", "t")
  res.register_embedding_dim("f", 4)
  t = ops.DenseCpuEmbeddingLookupTransform(res, "f", pad_value=0)
  dense = np.array([[1, 0, 2], [0, 0, 0], [3, 42, 0]], np.int64)
  with pytest.raises(xse.XseError) as e:
    t([dense])
  # CSR ids: [1, 2, 0 (all-pad row), 3, 42] -> 42 at index 4.
  assert e.value.message == ("FP32 embedding-bag request 0: Embedding ID (42) "
                             "at index 4 is out of bounds [0, 10).")
