"""GPU parity tests of the pooled lookup: the CUDA path (called through the C
ABI) against the CPU oracle on the same inputs. fp32-accumulated results are
compared bit for bit (the kernels keep the reference's CSR addition order and
rounding); error statuses and messages must match exactly."""

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import (TORCH_DT, assert_bitwise, assert_pooled,
                            expect_pool, oracle_pool,
                            random_csr, random_table, to_dev)

pytestmark = pytest.mark.gpu


def make_engine(xse, golden_tables):
  eng = xse.EmbeddingEngine(0)
  for name, t in golden_tables.items():
    data = np.asarray(t["data"], np.float32).reshape(-1, t["dim"])
    eng.add_table(name, data, t["combine"])
    eng.register_feature(name, name)
  return eng


def golden_requests(xse, case, outputs):
  reqs = []
  for r, out in zip(case["requests"], outputs):
    w = r.get("weights")
    reqs.append(xse.BagRequest(
        r["table"], to_dev(np.asarray(r["ids"], np.int64)),
        to_dev(np.asarray(r["offsets"], np.int32)), out,
        None if w is None else to_dev(np.asarray(w, np.float32))))
  return reqs


def test_golden_known_answers(xse, golden):
  for case in golden["cases"]:
    eng = make_engine(xse, case["tables"])
    if "requests" in case:
      outs = []
      for r in case["requests"]:
        dim = case["tables"][r["table"]]["dim"]
        outs.append(torch.full((len(r["offsets"]) - 1, dim), -99.0,
                               device="cuda"))
      eng.execute_batch(golden_requests(xse, case, outs))
      want = []
      for r in case["requests"]:
        t = case["tables"][r["table"]]
        want.append(oracle.embedding_bag(
            np.asarray(t["data"], np.float32).reshape(-1, t["dim"]), r["ids"],
            np.asarray(r["offsets"], np.int32), r.get("weights"),
            t["combine"]))
    else:
      outs, want = [], []
      for entry in case["dense"]:
        t = case["tables"][entry["table"]]
        ids, rp = oracle.dense_to_csr(np.asarray(entry["ids"], np.int32),
                                      entry["pad_value"])
        outs.append(eng.pool(entry["table"], to_dev(ids), to_dev(rp)))
        want.append(oracle.embedding_bag(
            np.asarray(t["data"], np.float32).reshape(-1, t["dim"]), ids, rp,
            combine=t["combine"]))
    for got, w, expect in zip(outs, want, case["expect"]):
      assert_bitwise(got.cpu().numpy(), w, case["name"])
      np.testing.assert_allclose(got.cpu().numpy().ravel(), expect,
                                 atol=case["tol"], rtol=0,
                                 err_msg=case["name"])
    eng.close()


@pytest.mark.parametrize("fused", [False, True])
def test_golden_errors(xse, golden, fused):
  for case in golden["errors"]:
    eng = make_engine(xse, case["tables"])
    outs = []
    shared = None
    weights_dev = {}
    reqs = []
    for k, r in enumerate(case["requests"]):
      dim = case["tables"][r["table"]]["dim"]
      nb = len(r["offsets"]) - 1
      w = r.get("weights")
      wd = None if w is None else to_dev(np.asarray(w, np.float32))
      weights_dev[k] = wd
      if r.get("output") == "shared":
        if shared is None:
          shared = torch.full((nb, dim), 23.0, device="cuda")
        out = shared
      elif r.get("output") == "weights":
        out = wd
      else:
        out = torch.full((nb, dim), 17.0 + k, device="cuda")
      outs.append(out)
      reqs.append(xse.BagRequest(
          r["table"], to_dev(np.asarray(r["ids"], np.int64)),
          to_dev(np.asarray(r["offsets"], np.int64)), out, wd))
    before = [o.clone() for o in outs]
    with pytest.raises(xse.XseError) as e:
      eng.execute_batch(reqs, fused=fused)
    assert e.value.code == case["code"], case["name"]
    assert e.value.message == case["message"], case["name"]
    if not fused:  # strict mode writes nothing on error
      for o, b in zip(outs, before):
        assert torch.equal(o, b), case["name"]
    eng.close()


DTYPES = [oracle.F32, oracle.BF16, oracle.I8_ROWWISE]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dim", [3, 16, 40, 64, 128, 256, 512])
@pytest.mark.parametrize("combine", ["SUM", "MEAN", "SQRT_N"])
def test_random_parity(xse, dtype, dim, combine):
  if dtype == oracle.I8_ROWWISE and dim == 3:
    dim = 5  # odd int8 rows still take the element-wise kernel
  rng = np.random.default_rng(dtype * 100003 + dim * 31 + len(combine))
  vocab = 300
  host, dev, scale, bias = random_table(rng, dtype, vocab, dim)
  eng = xse.EmbeddingEngine(0)
  eng.add_table("t", dev, combine, scale=scale, bias=bias)
  eng.register_feature("f", "t")
  for weighted in (False, True):
    for first in (0, 5):
      ids, offsets = random_csr(rng, vocab, 97, 70, first=first)
      w = rng.uniform(0, 1, len(ids)).astype(np.float32) if weighted else None
      for off_dt in (np.int32, np.int64):
        for id_dt in (torch.int32, torch.int64):
          got = eng.pool("f", to_dev(ids, id_dt), to_dev(offsets.astype(off_dt)),
                         None if w is None else to_dev(w))
          want = expect_pool(host, dtype, ids, offsets.astype(off_dt), w,
                             combine, scale, bias)
          assert_pooled(got.cpu().numpy(), want,
                         f"dtype={dtype} dim={dim} {combine} w={weighted} "
                         f"first={first}")
      got_fused = eng.pool("f", to_dev(ids), to_dev(offsets),
                           None if w is None else to_dev(w), fused=True)
      assert_pooled(got_fused.cpu().numpy(), want, "fused")
  eng.close()


def test_strided_output_and_mixed_group(xse):
  """One group mixing dtypes and dims, written into a [B, T, D] buffer like
  the DLRM pooled layout, and a second group into plain outputs."""
  rng = np.random.default_rng(11)
  eng = xse.EmbeddingEngine(0)
  specs = [(oracle.F32, 128, "SUM"), (oracle.BF16, 128, "MEAN"),
           (oracle.I8_ROWWISE, 128, "SQRT_N"), (oracle.F32, 128, "MEAN")]
  batch, hosts = 257, []
  for k, (dt, dim, comb) in enumerate(specs):
    host, dev, s, b = random_table(rng, dt, 1000 + k, dim)
    hosts.append((host, s, b))
    eng.add_table(f"t{k}", dev, comb, scale=s, bias=b)
    eng.register_feature(f"f{k}", f"t{k}")
  pooled = torch.full((batch, len(specs), 128), -1.0, device="cuda")
  reqs, want = [], []
  for k, (dt, dim, comb) in enumerate(specs):
    ids, offsets = random_csr(rng, 1000 + k, batch, 40)
    w = rng.uniform(0, 1, len(ids)).astype(np.float32) if k % 2 else None
    reqs.append(xse.BagRequest(f"f{k}", to_dev(ids), to_dev(offsets),
                               pooled[:, k, :], None if w is None else to_dev(w),
                               output_stride=len(specs) * 128))
    host, s, b = hosts[k]
    want.append(expect_pool(host, dt, ids, offsets, w, comb, s, b))
  eng.execute_batch(reqs)
  got = pooled.cpu().numpy()
  for k in range(len(specs)):
    assert_pooled(got[:, k, :], want[k], f"table {k}")
  # Interleaved column blocks are disjoint; overlapping ones are rejected
  # before anything is written.
  before = pooled.clone()
  reqs[3].output = pooled[:, 2, 64:].contiguous()  # separate buffer: fine
  reqs[3].output = pooled.view(batch, -1)[:, 2 * 128 + 64:]
  with pytest.raises(xse.XseError) as e:
    eng.execute_batch(reqs)
  assert e.value.message == "FP32 embedding-bag request outputs 2 and 3 overlap."
  assert torch.equal(pooled, before)
  eng.close()


def test_shard_windows_sum_to_whole(xse):
  """Row-wise shards: each engine holds a window of rows; ids outside it are
  skipped. The per-shard partials add up to the whole-table pool."""
  rng = np.random.default_rng(12)
  vocab, dim = 1000, 64
  host, dev, _, _ = random_table(rng, oracle.F32, vocab, dim)
  ids, offsets = random_csr(rng, vocab, 200, 30)
  whole = oracle_pool(host, oracle.F32, ids, offsets, None, "SUM")
  bounds = [0, 250, 600, 1000]
  total = np.zeros_like(whole, dtype=np.float64)
  for s in range(3):
    eng = xse.EmbeddingEngine(0)
    lo, hi = bounds[s], bounds[s + 1]
    eng.add_table("t", dev[lo:hi], "SUM", vocab=vocab, row_begin=lo,
                  row_end=hi)
    eng.register_feature("f", "t")
    part = eng.pool("f", to_dev(ids), to_dev(offsets)).cpu().numpy()
    keep = (ids >= lo) & (ids < hi)
    want = oracle_pool(host, oracle.F32, np.where(keep, ids, 0), offsets,
                       keep.astype(np.float32), "SUM")
    np.testing.assert_allclose(part, want, rtol=1e-6, atol=1e-6)
    total += part
    eng.close()
  np.testing.assert_allclose(total, whole, rtol=1e-5, atol=1e-5)


def test_async_status_and_errors(xse):
  rng = np.random.default_rng(13)
  host, dev, _, _ = random_table(rng, oracle.F32, 100, 32)
  eng = xse.EmbeddingEngine(0)
  eng.add_table("t", dev, "SUM")
  eng.register_feature("f", "t")
  eng.register_feature("seq", "t", max_sequence_length=4)
  ids, offsets = random_csr(rng, 100, 50, 10)
  out = torch.empty((50, 32), device="cuda")
  st = xse.Status(8)
  eng.execute_batch([xse.BagRequest("f", to_dev(ids), to_dev(offsets), out)],
                    status=st)
  st.wait()
  assert_bitwise(out.cpu().numpy(), oracle_pool(host, oracle.F32, ids, offsets,
                                                None, "SUM"))
  bad = ids.copy()
  bad[len(bad) // 2] = 100
  eng.execute_batch([xse.BagRequest("f", to_dev(bad), to_dev(offsets), out)],
                    status=st, fused=True)
  with pytest.raises(xse.XseError) as e:
    st.wait()
  assert e.value.message == (
      f"FP32 embedding-bag request 0: Embedding ID (100) at index "
      f"{len(bad) // 2} is out of bounds [0, 100).")
  with pytest.raises(xse.XseError) as e:
    eng.execute_batch([])
  assert e.value.message == "Embedding batch requires at least one request."
  with pytest.raises(xse.XseError) as e:
    eng.execute_batch([xse.BagRequest("nope", to_dev(ids), to_dev(offsets),
                                      out)])
  assert e.value.code == xse._capi.NOT_FOUND
  with pytest.raises(xse.XseError) as e:
    eng.execute_batch([xse.BagRequest("seq", to_dev(ids), to_dev(offsets),
                                      out)])
  assert e.value.code == xse._capi.UNIMPLEMENTED
  with pytest.raises(xse.XseError) as e:
    eng.add_table("t", dev, "SUM")
  assert e.value.code == xse._capi.ALREADY_EXISTS
  with pytest.raises(xse.XseError) as e:
    eng.register_feature("f", "t")
  assert e.value.code == xse._capi.ALREADY_EXISTS
  eng.clear()
  with pytest.raises(xse.XseError) as e:
    eng.pool("f", to_dev(ids), to_dev(offsets))
  assert e.value.code == xse._capi.NOT_FOUND
  st.close()
  eng.close()


def test_async_ring_reports_first_failure(xse):
  """Asynchronous executions share a status ring: the wait reports the first
  failing execution, including after the ring wrapped; the status is
  reusable after a wait, and a synchronous call settles pending ones."""
  rng = np.random.default_rng(21)
  host, dev, _, _ = random_table(rng, oracle.F32, 50, 16)
  eng = xse.EmbeddingEngine(0)
  eng.add_table("t", dev, "SUM")
  eng.register_feature("f", "t")
  ids, offsets = random_csr(rng, 50, 40, 6)
  good = to_dev(ids)
  bad_host = ids.copy()
  bad_host[3] = 50
  bad = to_dev(bad_host)
  offs = to_dev(offsets)
  out = torch.empty((40, 16), device="cuda")
  st = xse.Status(4)
  want = oracle_pool(host, oracle.F32, ids, offsets, None, "SUM")
  msg = ("FP32 embedding-bag request 0: Embedding ID (50) at index 3 is out "
         "of bounds [0, 50).")
  for failing in (10, 70):  # 70: the ring (64 slots) wraps first
    for k in range(100):
      eng.execute_batch([xse.BagRequest("f", bad if k == failing else good,
                                        offs, out)], status=st)
    with pytest.raises(xse.XseError) as e:
      st.wait()
    assert e.value.message == msg
    st.wait()  # settled: nothing pending
  for _ in range(3):
    eng.execute_batch([xse.BagRequest("f", good, offs, out)], status=st)
  st.wait()
  assert_bitwise(out.cpu().numpy(), want, "after ring")
  # A synchronous call through the same status block settles pending
  # asynchronous executions first and reports their error.
  eng.execute_batch([xse.BagRequest("f", bad, offs, out)], status=st)
  arr, _ = eng._c_requests([xse.BagRequest("f", good, offs, out)])
  rc = xse._capi.lib.xse_engine_execute_batch(
      eng.handle, arr, 1, xse.stream_handle(), xse._capi.EXEC_STRICT,
      st.handle)
  assert rc == xse._capi.INVALID_ARGUMENT
  assert xse._capi.last_error() == msg
  rc = xse._capi.lib.xse_engine_execute_batch(
      eng.handle, arr, 1, xse.stream_handle(), xse._capi.EXEC_STRICT,
      st.handle)
  assert rc == xse._capi.OK
  st.close()
  eng.close()


def test_addition_order_fixture(xse):
  import os  # pylint: disable=import-outside-toplevel
  g = np.load(os.path.join(os.path.dirname(__file__), "golden",
                           "numpy_lookup.npz"))
  eng = xse.EmbeddingEngine(0)
  eng.add_table("t", g["order_table"], "SUM")
  eng.register_feature("f", "t")
  got = eng.pool("f", to_dev(g["order_ids"]), to_dev(g["order_offsets"]))
  assert_bitwise(got.cpu().numpy(), g["order_out"], "order")
  for i in range(int(g["num_tables"])):
    eng.add_table(f"n{i}", g[f"table_{i}"], "SUM")
    eng.register_feature(f"n{i}", f"n{i}")
    dense = g[f"ids_{i}"]
    b, v = dense.shape
    offs = np.arange(b + 1, dtype=np.int32) * v
    got = eng.pool(f"n{i}", to_dev(dense.ravel()), to_dev(offs)).cpu().numpy()
    want = oracle.embedding_bag(g[f"table_{i}"], dense.ravel(), offs)
    assert_bitwise(got, want, f"numpy fixture {i}")
    np.testing.assert_allclose(got, g[f"out_{i}"], rtol=1e-5, atol=1e-6)
  eng.close()


def test_dtype_table_views(xse):
  assert TORCH_DT[oracle.BF16] == torch.bfloat16
  eng = xse.EmbeddingEngine(0)
  eng.add_table("t", np.zeros((4, 8), np.float32), "MEAN")
  info = eng.table_info("t")
  assert (info.vocab, info.dim, info.combine) == (4, 8, 2)
  eng.close()


@pytest.mark.parametrize("dtype,dim", [(oracle.F32, 64), (oracle.BF16, 128),
                                       (oracle.F32, 128), (oracle.BF16, 64)])
def test_large_launch_parity(xse, dtype, dim):
  """Small launches take the staged kernel (rows copied to shared memory);
  large ones the throughput kernel or the staged one, whichever the engine's
  tuner measures faster -- its first executions of a launch alternate the
  two. Every kernel must give the oracle's bits: a 16,000-bag batch
  (weighted mean and plain sum), run six times (both kernels, then the
  chosen one), against the small-batch result of the same bags."""
  rng = np.random.default_rng(dim + 7 * dtype)
  vocab = 50_000
  host, dev, scale, bias = random_table(rng, dtype, vocab, dim)
  eng = xse.EmbeddingEngine(0)
  for combine in ("SUM", "MEAN"):
    eng.add_table(f"t_{combine}", dev, combine)
    eng.register_feature(f"f_{combine}", f"t_{combine}")
  ids, offsets = random_csr(rng, vocab, 16_000, 30)
  w = rng.uniform(0, 1, len(ids)).astype(np.float32)
  for combine, weights in (("SUM", None), ("MEAN", w)):
    want = oracle_pool(host, dtype, ids, offsets, weights, combine, scale,
                       bias)
    d_ids, d_offsets = to_dev(ids), to_dev(offsets)
    d_w = None if weights is None else to_dev(weights)
    for run in range(6):
      got = eng.pool(f"f_{combine}", d_ids, d_offsets, d_w)
      assert_bitwise(got.cpu().numpy(), want, f"large {combine} run {run}")
    # The first 200 bags alone (a small launch) give the same rows.
    small = eng.pool(f"f_{combine}", to_dev(ids), to_dev(offsets[:201]),
                     None if weights is None else to_dev(weights))
    assert_bitwise(small.cpu().numpy(), want[:200], f"small {combine}")
  eng.close()


@pytest.mark.parametrize("id_dtype", [np.int64, np.int32])
@pytest.mark.parametrize("skew", [0, 1, 3])
def test_validation_reports_smallest_bad_position(xse, id_dtype, skew):
  """The id check reads 16-byte vectors when the ids are aligned and single
  ids otherwise (`skew` shifts the ids off alignment); either way the
  reported position is the smallest failing one inside [offsets[0],
  offsets[-1]), and ids outside that range are not read."""
  rng = np.random.default_rng(41 + skew)
  _, dev, _, _ = random_table(rng, oracle.F32, 1000, 32)
  eng = xse.EmbeddingEngine(0)
  eng.add_table("t", dev, "SUM")
  eng.register_feature("f", "t")
  n = 9000
  ids = rng.integers(0, 1000, size=n + skew).astype(id_dtype)
  backing = to_dev(ids)
  view = backing[skew:]
  lens = rng.integers(0, 9, size=2000)
  first = 5
  offsets = np.concatenate([[first], first + np.cumsum(lens)])
  offsets = offsets[offsets <= n - 7]
  out = torch.empty((len(offsets) - 1, 32), device="cuda")
  last = int(offsets[-1])
  for bad_positions in ([first], [last - 1], [2049, 2050, 7000],
                        [4097, 4096 + 2], [first + 1, first + 3]):
    host = ids.copy()
    host[skew:][:first] = -1            # before offsets[0]: not read
    host[skew:][last:] = 1000           # at or past offsets[-1]: not read
    for pos in bad_positions:
      if pos < last:
        host[skew + pos] = 1000 + pos
    backing.copy_(torch.from_numpy(host))
    expect = min(p for p in bad_positions if p < last)
    with pytest.raises(xse.XseError) as e:
      eng.execute_batch([xse.BagRequest("f", view, to_dev(
          offsets.astype(np.int64)), out)])
    assert e.value.message == (
        f"FP32 embedding-bag request 0: Embedding ID ({1000 + expect}) at "
        f"index {expect} is out of bounds [0, 1000).")
  host = ids.copy()
  host[skew:][:first] = -1
  host[skew:][last:] = 1000
  backing.copy_(torch.from_numpy(host))
  eng.execute_batch([xse.BagRequest("f", view, to_dev(
      offsets.astype(np.int64)), out)])
  eng.close()


def test_profiling_period(xse):
  """Kernel timing samples every `period`-th execution and counts all."""
  rng = np.random.default_rng(5)
  _, dev, _, _ = random_table(rng, oracle.F32, 100, 32)
  eng = xse.EmbeddingEngine(0)
  eng.add_table("t", dev, "SUM")
  eng.register_feature("f", "t")
  ids, offsets = random_csr(rng, 100, 64, 6)
  reqs = [xse.BagRequest("f", to_dev(ids), to_dev(offsets),
                         torch.empty((64, 32), device="cuda"))]
  eng.set_profiling(True, 3)
  for _ in range(7):
    eng.execute_batch(reqs)
  ms, timed, calls = eng.profile_read(with_calls=True)
  assert (timed, calls) == (3, 7) and ms > 0
  eng.execute_batch(reqs)  # the read restarts the sampling: timed
  ms, timed = eng.profile_read()
  assert timed == 1
  # Strict executions run the validation kernel, fused ones do not.
  eng.set_profiling(True, 1)
  eng.execute_batch(reqs)
  eng.execute_batch(reqs, fused=True)
  st = eng.profile_read_stages()
  assert (st["executions"], st["validated"], st["calls"]) == (2, 1, 2)
  assert st["validate_ms"] > 0 and st["pool_ms"] > 0
  eng.set_profiling(False)
  eng.execute_batch(reqs)
  assert eng.profile_read(with_calls=True)[1:] == (0, 0)
  with pytest.raises(xse.XseError):
    C = xse._capi
    C.check(C.lib.xse_engine_set_profiling(eng._handle, -1))
  eng.close()


@pytest.mark.parametrize("dtype,dim", [(oracle.BF16, 128), (oracle.I8_ROWWISE,
                                                            256),
                                       (oracle.BF16, 64)])
@pytest.mark.parametrize("shift", [0, 4, 1])
def test_output_alignment_variants(xse, dtype, dim, shift):
  """Lanes store 32-byte pieces only where the output row is 32-byte
  aligned: rows shifted by 4 floats (16-byte aligned) take 16-byte stores,
  rows shifted by 1 float scalar stores. All three match the oracle bit for
  bit and leave the floats around every row untouched."""
  rng = np.random.default_rng(100 + dim + shift)
  eng = xse.EmbeddingEngine(0)
  vocab, batch = 900, 131
  host, dev, s, b = random_table(rng, dtype, vocab, dim)
  eng.add_table("t", dev, "MEAN", scale=s, bias=b)
  eng.register_feature("f", "t")
  ids, offsets = random_csr(rng, vocab, batch, 37)
  w = rng.uniform(0, 1, len(ids)).astype(np.float32)
  stride = dim + 8 + (shift % 4)  # keeps every row at the same alignment
  buf = torch.full((batch * stride + 16,), -3.0, device="cuda")
  out = buf[shift:shift + batch * stride].view(batch, stride)[:, :dim]
  eng.execute_batch([xse.BagRequest("f", to_dev(ids), to_dev(offsets), out,
                                    to_dev(w), output_stride=stride)])
  want = expect_pool(host, dtype, ids, offsets, w, "MEAN", s, b)
  assert_pooled(out.cpu().numpy(), want, f"shift {shift}")
  rest = buf.clone()
  rest[shift:shift + batch * stride].view(batch, stride)[:, :dim] = -3.0
  assert torch.all(rest == -3.0)
  eng.close()
