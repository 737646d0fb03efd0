"""GPU tests of the legacy per-feature path (xse_engine_execute_legacy,
CpuEmbeddingEngine::Execute): pooling in the table's type (fp32 as the
batched path, bf16 accumulating in bf16) and sequence gathers, against the
oracle bit for bit and against the reference's own known answers;
FeatureBatchCsrInput and bounds errors with the reference's messages."""

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import random_csr, to_dev

pytestmark = pytest.mark.gpu


def bf16_bits(a):
  """fp32 -> bf16 bits, rounded to nearest even (as Eigen's bfloat16(x))."""
  u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
  return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def engine_with(xse, tables, sequences=None):
  """tables: name -> (host array fp32 or bf16 bits, combine)."""
  eng = xse.EmbeddingEngine(0)
  for name, (data, combine) in tables.items():
    eng.add_table(name, data, combine)
    seq = (sequences or {}).get(name, 0)
    eng.register_feature(name, name, seq)
  return eng


@pytest.mark.parametrize("combine", ["SUM", "MEAN", "SQRT_N"])
@pytest.mark.parametrize("weighted", [False, True])
def test_pooled_fp32_and_bf16(xse, combine, weighted):
  rng = np.random.default_rng(len(combine) + 10 * weighted)
  vocab, dim = 500, 40
  f32 = rng.uniform(-1, 1, (vocab, dim)).astype(np.float32)
  b16 = bf16_bits(rng.uniform(-1, 1, (vocab, dim)))
  eng = engine_with(xse, {"f": (f32, combine), "b": (b16, combine)})
  ids, offsets = random_csr(rng, vocab, 300, 25)
  rp = offsets.astype(np.int32)
  w = rng.uniform(0.1, 1, len(ids)).astype(np.float32) if weighted else None
  reqs = [xse.BagRequest(name, to_dev(ids), to_dev(rp), None,
                         None if w is None else to_dev(w))
          for name in ("f", "b")]
  got_f, got_b = eng.execute_legacy(reqs)
  assert got_f.dtype == torch.float32 and got_b.dtype == torch.bfloat16
  np.testing.assert_array_equal(
      got_f.cpu().numpy(), oracle.embedding_bag(f32, ids, rp, w, combine))
  want_b = oracle.assemble_bf16_accumulate(b16, ids, rp, w, combine)
  np.testing.assert_array_equal(
      got_b.cpu().view(torch.int16).numpy().view(np.uint16), want_b)
  eng.close()


@pytest.mark.parametrize("bf16", [False, True])
def test_sequence_gather(xse, golden, bf16):
  case = golden["sequence"][0]
  table = (np.arange(40, dtype=np.float32) * np.float32(0.1)).reshape(10, 4)
  data = bf16_bits(table) if bf16 else table
  eng = engine_with(xse, {"t": (data, "SUM")}, {"t": 5})
  out, = eng.execute_legacy([xse.BagRequest(
      "t", to_dev(np.array(case["ids"], np.int64)),
      to_dev(np.array(case["offsets"], np.int32)), None)])
  assert out.shape == (3, 5, 4)
  got = out.float().cpu().numpy().ravel()
  tol = case["bf16_tol"] if bf16 else case["tol"]
  np.testing.assert_allclose(got, case["expect"], rtol=0, atol=tol)
  want = oracle.sequence_gather(data, case["ids"], case["offsets"], 5,
                                oracle.BF16 if bf16 else oracle.F32)
  raw = out.cpu()
  raw = raw.view(torch.int16).numpy().view(np.uint16) if bf16 else raw.numpy()
  np.testing.assert_array_equal(raw, want)
  eng.close()


def test_sequence_truncates_and_mixes_with_pooled(xse):
  rng = np.random.default_rng(4)
  vocab, dim = 300, 16
  table = rng.standard_normal((vocab, dim)).astype(np.float32)
  eng = engine_with(xse, {"seq": (table, "SUM"), "pool": (table, "MEAN")},
                    {"seq": 7})
  ids, offsets = random_csr(rng, vocab, 200, 20)
  rp = offsets.astype(np.int32)
  long_bag = int(np.argmax(np.diff(rp) >= 9))
  assert rp[long_bag + 1] - rp[long_bag] >= 9
  ids[rp[long_bag] + 8] = 99999  # past max_sequence_length: never checked
  seq, pooled = eng.execute_legacy([
      xse.BagRequest("seq", to_dev(ids), to_dev(rp), None),
      xse.BagRequest("pool", to_dev(np.where(ids < vocab, ids, 0)),
                     to_dev(rp), None)])
  np.testing.assert_array_equal(
      seq.cpu().numpy(), oracle.sequence_gather(table, ids, rp, 7))
  np.testing.assert_array_equal(
      pooled.cpu().numpy(),
      oracle.embedding_bag(table, np.where(ids < vocab, ids, 0), rp, None,
                           "MEAN"))
  eng.close()


def test_errors(xse):
  table = np.ones((10, 4), np.float32)
  eng = engine_with(xse, {"t": (table, "SUM"), "s": (table, "SUM")}, {"s": 3})

  def run(name, ids, rp, w=None):
    with pytest.raises(xse.XseError) as e:
      eng.execute_legacy([xse.BagRequest(
          name, to_dev(np.array(ids, np.int64)),
          to_dev(np.array(rp, np.int32)), None,
          None if w is None else to_dev(np.array(w, np.float32)))])
    return e.value

  # FeatureBatchCsrInput (feature_batch_csr_input.cc:36-54)
  e = run("t", [1, 2], [1, 2])
  assert e.message == ("Embedding ids size (2) does not match last element "
                       "of row pointers (2)")
  e = run("t", [1, 2, 3], [0, 3, 2, 3])
  assert e.message == "Row pointers are not sorted."
  e = run("t", [1, 2], [0, 2], [1.0])
  assert e.message == "Weights size (1) does not match expected size (2)"
  e = run("t", [1], [0])
  assert e.message == "Row pointers must have at least 2 elements."
  # Bounds (compute_activations.cc:89-98): index in the batch.
  e = run("t", [1, 2, 3, 11], [0, 2, 4])
  assert e.message == ("Embedding ID (11) at index 3 is out of bounds "
                       "[0, 10) for table t.")
  # Sequence (compute_activations.cc:205-213): index in the sample.
  e = run("s", [1, 2, 3, 11], [0, 2, 4])
  assert e.message == ("Embedding ID (11) at index 1 is out of bounds "
                       "[0, 10) for table s.")
  e = run("s", [1, 2], [0, 2], [1.0, 1.0])
  assert e.message == "Weights should be empty for sequence assembly."
  e = run("missing", [1], [0, 1])
  assert e.code == xse._capi.NOT_FOUND
  assert e.message == "Feature spec not found for: missing"
  eng.close()
