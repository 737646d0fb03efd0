"""CPU tests of the oracle against the reference's golden vectors.

Pins the C++ restatement (oracle/xse_oracle.cc) before the CUDA path is
tested against it: every known answer of the reference's tests
(tests/golden/known_answers.json) and the reference's numpy lookup run on
seeded inputs (tests/golden/numpy_lookup.npz).
"""

import os

import numpy as np
import pytest

from oracle import oracle

GOLDEN_NPZ = os.path.join(os.path.dirname(__file__), "golden",
                          "numpy_lookup.npz")


def table_array(spec):
  return np.asarray(spec["data"], dtype=np.float32).reshape(-1, spec["dim"])


def run_case_requests(case, num_threads=1):
  bags = []
  for r in case["requests"]:
    t = case["tables"][r["table"]]
    bags.append(oracle.Bag(table_array(t), r["ids"],
                           np.asarray(r["offsets"], dtype=np.int32),
                           r.get("weights"), t["combine"]))
  return oracle.embedding_bag_batch(bags, num_threads=num_threads,
                                    inline_threshold=0)


def dense_case(case, entry):
  t = case["tables"][entry["table"]]
  ids, rp = oracle.dense_to_csr(np.asarray(entry["ids"], dtype=np.int32),
                                entry["pad_value"])
  out = oracle.embedding_bag(table_array(t), ids, rp, combine=t["combine"])
  return ids, rp, out


@pytest.mark.parametrize("threads", [1, 3])
def test_known_answers(golden, threads):
  for case in golden["cases"]:
    if "requests" in case:
      outs = run_case_requests(case, threads)
    else:
      outs = [dense_case(case, e)[2] for e in case["dense"]]
    for got, want in zip(outs, case["expect"]):
      np.testing.assert_allclose(got.ravel(), np.asarray(want, np.float32),
                                 rtol=0, atol=max(case["tol"], 0),
                                 err_msg=case["name"])


def test_dense_all_pad_csr(golden):
  case = next(c for c in golden["cases"]
              if c["name"] == "dense_all_padded_keeps_one_pad_id")
  ids, rp, _ = dense_case(case, case["dense"][0])
  assert ids.tolist() == case["csr"]["ids"]
  assert rp.tolist() == case["csr"]["row_pointers"]


def test_known_errors(golden):
  for case in golden["errors"]:
    bags = []
    shared = None
    for r in case["requests"]:
      t = case["tables"][r["table"]]
      table = table_array(t)
      bag = oracle.Bag(table, r["ids"], np.asarray(r["offsets"], np.int64),
                       r.get("weights"), t["combine"])
      if r.get("output") == "shared":
        if shared is None:
          shared = np.zeros_like(bag.out)
        bag.out = shared
      elif r.get("output") == "weights":
        bag.out = bag.weights.reshape(1, -1)
      bags.append(bag)
    snapshot = [b.out.copy() for b in bags]
    with pytest.raises(oracle.OracleError) as e:
      oracle.embedding_bag_batch(bags)
    assert e.value.code == case["code"], case["name"]
    assert e.value.message == case["message"], case["name"]
    for b, before in zip(bags, snapshot):
      np.testing.assert_array_equal(b.out, before)  # no partial writes


def test_dense_row_pointer_errors(golden):
  for case in golden["dense_row_pointer_errors"]:
    with pytest.raises(oracle.OracleError) as e:
      oracle.dense_lookup_row_pointers(case["batch"], case["valency"],
                                       materialize=False)
    assert case["message"] in e.value.message
  rp = oracle.dense_lookup_row_pointers(3, 4)
  assert rp.tolist() == [0, 4, 8, 12]


def test_reference_numpy_lookup_fixture():
  """The reference's own numpy lookup (examples/dlrm_benchmark/common.py)
  on seeded inputs; numpy sums pairwise, so compare within fp32 rounding."""
  g = np.load(GOLDEN_NPZ)
  for i in range(int(g["num_tables"])):
    table = g[f"table_{i}"]
    dense = g[f"ids_{i}"]
    batch, valency = dense.shape
    offsets = np.arange(batch + 1, dtype=np.int32) * valency
    out = oracle.embedding_bag(table, dense.ravel(), offsets)
    want = g[f"out_{i}"]
    bound = 4 * np.finfo(np.float32).eps * valency * np.abs(
        table[dense]).sum(axis=1)
    assert np.all(np.abs(out - want) <= bound + 1e-12), i


def test_addition_order_is_csr_order():
  """embedding_bag_test.cc:296-343: +-1e20 rows expose the summation order;
  the oracle must match the strict CSR-order fp32 sum bit for bit."""
  g = np.load(GOLDEN_NPZ)
  out = oracle.embedding_bag(g["order_table"], g["order_ids"],
                             g["order_offsets"])
  np.testing.assert_array_equal(out, g["order_out"])
  threaded = oracle.embedding_bag(g["order_table"], g["order_ids"],
                                  g["order_offsets"], num_threads=4)
  np.testing.assert_array_equal(threaded, g["order_out"])


def test_bf16_accumulate_known_answers(golden):
  """The reference's bf16 path (bf16 accumulator) meets its own 1e-2
  tolerance on the compute_activations known answers."""
  for case in golden["cases"]:
    if "bf16_tol" not in case:
      continue
    r = case["requests"][0]
    t = case["tables"][r["table"]]
    f32 = table_array(t)
    bits = (f32.view(np.uint32) + 0x7FFF + ((f32.view(np.uint32) >> 16) & 1)
            ) >> 16
    out = oracle.assemble_bf16_accumulate(bits.astype(np.uint16), r["ids"],
                                          r["offsets"], r.get("weights"),
                                          t["combine"])
    got = oracle.bf16_bits_to_f32(out).ravel()
    np.testing.assert_allclose(got, case["expect"][0], atol=case["bf16_tol"])


def test_threaded_matches_inline_bitwise():
  rng = np.random.default_rng(7)
  table = rng.uniform(-0.05, 0.05, (5000, 64)).astype(np.float32)
  lengths = rng.integers(0, 40, 3000)
  offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
  ids = rng.integers(0, 5000, offsets[-1])
  w = rng.uniform(0, 1, offsets[-1]).astype(np.float32)
  for combine in ("SUM", "MEAN", "SQRT_N"):
    for weights in (None, w):
      a = oracle.embedding_bag(table, ids, offsets, weights, combine)
      b = oracle.embedding_bag(table, ids, offsets, weights, combine,
                               num_threads=5)
      np.testing.assert_array_equal(a, b)


def test_int8_and_bf16_widening():
  rng = np.random.default_rng(3)
  q = rng.integers(-127, 128, (50, 32)).astype(np.int8)
  scale = rng.uniform(1e-3, 1e-2, 50).astype(np.float32)
  bias = rng.uniform(-0.1, 0.1, 50).astype(np.float32)
  ids = rng.integers(0, 50, 40)
  offsets = np.array([0, 10, 10, 25, 40], dtype=np.int64)
  got = oracle.embedding_bag(q, ids, offsets, dtype=oracle.I8_ROWWISE,
                             scale=scale, bias=bias)
  # Dequantized to an fp32 row first: float(q) * scale rounded to fp32,
  # then + bias rounded to fp32 (numpy float32 arithmetic rounds each
  # operation), then the fp32 bag.
  deq = (q.astype(np.float32) * scale[:, None]) + bias[:, None]
  assert deq.dtype == np.float32
  want = np.zeros_like(got)
  for b in range(4):
    for p in range(offsets[b], offsets[b + 1]):
      want[b] = (want[b] + deq[ids[p]]).astype(np.float32)
  np.testing.assert_array_equal(got, want)

  f32 = rng.uniform(-1, 1, (50, 32)).astype(np.float32)
  bits = (f32.view(np.uint32) >> 16).astype(np.uint16)
  got = oracle.embedding_bag(bits, ids, offsets, dtype=oracle.BF16)
  widened = oracle.bf16_bits_to_f32(bits).reshape(50, 32)
  want = oracle.embedding_bag(widened, ids, offsets)
  np.testing.assert_array_equal(got, want)


def test_absolute_offsets_and_empty_bags():
  table = np.arange(12, dtype=np.float32).reshape(4, 3)
  ids = np.array([3, 3, 0, 1, 2], dtype=np.int64)
  offsets = np.array([2, 2, 4, 5], dtype=np.int64)  # front() > 0
  out = oracle.embedding_bag(table, ids, offsets)
  np.testing.assert_array_equal(out, [[0, 0, 0], [3, 5, 7], [6, 7, 8]])


def test_dot_interaction_small():
  rng = np.random.default_rng(5)
  dense = rng.normal(size=(3, 8)).astype(np.float32)
  pooled = rng.normal(size=(3, 4, 8)).astype(np.float32)
  out = oracle.dot_interaction(dense, pooled)
  assert out.shape == (3, 8 + 10)
  for b in range(3):
    z = np.concatenate([dense[b:b + 1], pooled[b]], axis=0).astype(np.float64)
    g = z @ z.T
    iu = np.triu_indices(5, k=1)
    np.testing.assert_allclose(out[b, 8:], g[iu], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(out[b, :8], dense[b])


def test_synth_rows_deterministic_and_in_range():
  a, _, _ = oracle.synth_rows(oracle.F32, 0, 0, 10, 5, 64)
  b, _, _ = oracle.synth_rows(oracle.F32, 0, 0, 12, 3, 64)
  np.testing.assert_array_equal(a[2:5], b)
  assert a.min() >= -0.05 and a.max() < 0.05
  q, s, bias = oracle.synth_rows(oracle.I8_ROWWISE, 0, 3, 0, 100, 256)
  assert q.min() >= -127 and q.max() <= 127
  assert s.min() >= 1e-3 and s.max() < 1e-2
  assert bias.min() >= -0.1 and bias.max() < 0.1
  bits, _, _ = oracle.synth_rows(oracle.BF16, 0, 0, 10, 5, 64)
  np.testing.assert_allclose(oracle.bf16_bits_to_f32(bits).reshape(5, 64), a,
                             rtol=1e-2)


def test_zipf_rank_distribution():
  n, alpha = 1000, 1.05
  ranks = np.array([oracle.zipf_rank(0, 2, i, n, alpha) for i in range(20000)])
  assert ranks.min() >= 1 and ranks.max() <= n
  counts = np.bincount(ranks, minlength=n + 1)[1:]
  p = np.arange(1, n + 1, dtype=np.float64) ** -alpha
  p /= p.sum()
  # Top ranks follow the Zipf law within sampling noise.
  for k in range(5):
    expected = p[k] * len(ranks)
    assert abs(counts[k] - expected) < 5 * np.sqrt(expected), k


def test_sequence_gather_known_answer(golden):
  """The oracle's AssembleSequenceEmbeddings against the reference test."""
  case = golden["sequence"][0]
  table = (np.arange(40, dtype=np.float32) * np.float32(0.1)).reshape(10, 4)
  got = oracle.sequence_gather(table, case["ids"], case["offsets"],
                               case["max_sequence_length"])
  assert got.shape == (3, 5, 4)
  np.testing.assert_allclose(got.ravel(), case["expect"], rtol=0,
                             atol=case["tol"])
  with pytest.raises(oracle.OracleError, match=r"\(12\) at index 1 "):
    oracle.sequence_gather(table, [1, 12, 4], [0, 2, 3], 5)
  # Ids past max_sequence_length are neither read nor checked.
  got = oracle.sequence_gather(table, [1, 3, 99], [0, 3], 2)
  np.testing.assert_array_equal(got[0], table[[1, 3]])
