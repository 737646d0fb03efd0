"""GPU tests of the synthetic-data kernels (bit-exact against the oracle's
independent restatement of the generator) and of the DLRM dot interaction
(against the oracle within 1e-4, condition-aware)."""

import math

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import assert_bitwise

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [oracle.F32, oracle.BF16, oracle.I8_ROWWISE])
def test_synth_table_matches_oracle(xse, dtype):
  from xla_serving_b200 import synth  # pylint: disable=import-outside-toplevel
  rows, scale, bias = synth.synth_table(dtype, 5000, 128, seed=0, table=3,
                                        row0=1234, nrows=300)
  want, ws, wb = oracle.synth_rows(dtype, 0, 3, 1234, 300, 128)
  if dtype == oracle.F32:
    assert_bitwise(rows.cpu().numpy(), want)
  elif dtype == oracle.BF16:
    got = rows.cpu().view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(got, want)
  else:
    np.testing.assert_array_equal(rows.cpu().numpy(), want)
    assert_bitwise(scale.cpu().numpy(), ws)
    assert_bitwise(bias.cpu().numpy(), wb)


def test_synth_ids_zipf_matches_oracle(xse):
  from xla_serving_b200 import synth  # pylint: disable=import-outside-toplevel
  vocab, n, alpha = 1_000_000, 4000, 1.05
  ids = synth.synth_ids(n, vocab, seed=0, table=7, zipf_alpha=alpha).cpu()
  mul = synth.coprime_multiplier(vocab)
  want = []
  for i in range(n):
    k = oracle.zipf_rank(0, 7 * 16 + 2, i, vocab, alpha)
    want.append(((k - 1) * mul + synth.PERM_ADD % vocab) % vocab)
  same = (ids.numpy() == np.array(want)).mean()
  # Device and host transcendentals may differ in the last ulp, which can
  # flip a rejection decision; that is vanishingly rare.
  assert same >= 0.999, same
  assert ids.min() >= 0 and ids.max() < vocab


def test_synth_lengths_and_uniform_ids(xse):
  from xla_serving_b200 import synth  # pylint: disable=import-outside-toplevel
  lengths = synth.synth_lengths(100000, 1, 32, seed=0, table=0).cpu().numpy()
  assert lengths.min() == 1 and lengths.max() == 32
  assert abs(lengths.mean() - 16.5) < 0.2
  ids = synth.synth_ids(100000, 777, seed=0, table=0).cpu().numpy()
  assert ids.min() >= 0 and ids.max() < 777
  counts = np.bincount(ids, minlength=777)
  assert counts.min() > 50
  w = synth.synth_weights(1000, seed=0, table=0).cpu().numpy()
  assert w.min() >= 0 and w.max() < 1


def check_interaction(got, dense, pooled):
  want = oracle.dot_interaction(dense, pooled)
  b, t, d = pooled.shape
  z = np.concatenate([dense[:, None, :], pooled], axis=1).astype(np.float64)
  iu = np.triu_indices(t + 1, k=1)
  mag = np.einsum("bic,bjc->bij", np.abs(z), np.abs(z))[:, iu[0], iu[1]]
  assert got.shape == want.shape
  np.testing.assert_array_equal(got[:, :d], want[:, :d])
  err = np.abs(got[:, d:].astype(np.float64) - want[:, d:])
  assert np.all(err <= 1e-4 * mag + 1e-7), float((err / (mag + 1e-30)).max())


@pytest.mark.parametrize("shape", [(1000, 26, 128), (33, 26, 128),
                                   (17, 5, 24), (8, 3, 7)])
def test_dot_interaction_matches_oracle(xse, shape):
  b, t, d = shape
  rng = np.random.default_rng(b * 7 + t)
  dense = rng.normal(size=(b, d)).astype(np.float32)
  pooled = rng.uniform(-0.05, 0.05, size=(b, t, d)).astype(np.float32) * 20
  got = xse.dot_interaction(torch.from_numpy(dense).cuda(),
                            torch.from_numpy(pooled).cuda())
  torch.cuda.synchronize()
  assert got.shape == (b, d + (t + 1) * t // 2)
  check_interaction(got.cpu().numpy(), dense, pooled)


def test_dot_interaction_dlrm_width(xse):
  assert 128 + 27 * 26 // 2 == 479
  dense = torch.zeros((2, 128), device="cuda")
  pooled = torch.ones((2, 26, 128), device="cuda")
  out = xse.dot_interaction(dense, pooled)
  assert out.shape == (2, 479)
  # pairs (0, j) involve the zero dense row; the rest are dot(1, 1) = 128.
  o = out.cpu().numpy()
  assert np.all(o[:, 128:128 + 26] == 0)
  assert np.all(o[:, 128 + 26:] == 128)
  assert math.isclose(float(o.sum()), 2 * 128 * (351 - 26))
