"""GPU tests of the pooled lookup fused with the dot interaction
(xse_engine_execute_interaction). The fused result is compared with the
unfused path on the same inputs -- execute_batch into a pooled [B, T, dim]
buffer (bit-exact to the oracle), then xse_dot_interaction_strided -- and
with the oracle directly:

* the dense columns and the zero pad match exactly;
* each dot product lies within 1e-5 of the unfused one, relative to
  sum_c |z_i,c z_j,c| (both are fp32 FMA chains, summed in different orders);
* with one-hot dense rows, the pair (dense, table t) of sample b is
  pooled[b, t, c_b] carried through the split-TF32 products (hi + lo parts,
  within 2^-20 relative), so the pooled rows inside the fused kernel are
  checked element by element against the oracle's.

Layouts with a fused kernel (fp32 / bf16 rows of 32 16-byte vectors, one
weighting mode, up to 31 tables) and layouts served by the unfused fallback
inside the same call are both covered."""

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import (assert_bitwise, oracle_pool, random_csr,
                            random_table, to_dev)

pytestmark = pytest.mark.gpu

# (dtype, dim, tables, batch, combine, weighting) -- weighting: None (no
# weights), "all" (every request weighted) or "mixed" (odd requests only).
CASES = [
    (oracle.F32, 128, 26, 37, "SUM", None),     # the DLRM layout (fused)
    (oracle.F32, 128, 26, 5000, "SUM", None),   # many samples per block:
                                                # shared-memory slots reused
    (oracle.F32, 128, 7, 41, "MEAN", "all"),    # fused, weighted mean
    (oracle.F32, 128, 9, 23, "SUM", "all"),     # fused, weighted sum
    (oracle.BF16, 256, 3, 9, "SQRTN", None),    # fused, bf16 rows
    (oracle.F32, 128, 31, 11, "SUM", None),     # fused, 32 rows in the Gram
    (oracle.F32, 64, 5, 50, "MEAN", "all"),     # 16-vector rows: fallback
    (oracle.BF16, 128, 8, 33, "SUM", "all"),    # 16-vector rows: fallback
    (oracle.F32, 40, 4, 20, "SUM", None),       # 10-vector rows: fallback
    (oracle.F32, 128, 6, 17, "SUM", "mixed"),   # two modes: fallback
    (oracle.F32, 128, 32, 7, "SUM", None),      # 33 rows: fallback
    (oracle.F32, 128, 1, 5, "MEAN", None),      # one table
]


def build(xse, rng, dtype, dim, tables, batch, combine, weighting):
  eng = xse.EmbeddingEngine(0)
  hosts, reqs, meta = [], [], []
  for t in range(tables):
    vocab = int(rng.integers(50, 400))
    host, dev, _, _ = random_table(rng, dtype, vocab, dim)
    eng.add_table(f"t{t}", dev, combine)
    eng.register_feature(f"f{t}", f"t{t}")
    ids, offsets = random_csr(rng, vocab, batch, 12, first=int(t % 3))
    weighted = weighting == "all" or (weighting == "mixed" and t % 2 == 1)
    w = (rng.uniform(0.1, 1.0, len(ids)).astype(np.float32)
         if weighted else None)
    hosts.append(host)
    meta.append((ids, offsets, w))
    reqs.append(xse.BagRequest(f"f{t}", to_dev(ids), to_dev(offsets), None,
                               None if w is None else to_dev(w)))
  return eng, hosts, reqs, meta


def unfused(xse, eng, reqs, dense, tables, dim, out_stride):
  batch = dense.shape[0]
  pooled = torch.empty((batch, tables, dim), device="cuda")
  eng.execute_batch([
      xse.BagRequest(r.feature_name, r.ids, r.offsets, pooled[:, k, :],
                     r.weights, output_stride=tables * dim)
      for k, r in enumerate(reqs)])
  out = torch.empty((batch, out_stride), device="cuda")
  C = xse._capi
  C.check(C.lib.xse_dot_interaction_strided(
      dense.data_ptr(), dense.stride(0), pooled.data_ptr(), pooled.stride(0),
      batch, tables, dim, out.data_ptr(), out.stride(0), None))
  torch.cuda.synchronize()
  return pooled.cpu().numpy(), out.cpu().numpy()


@pytest.mark.parametrize("dtype,dim,tables,batch,combine,weighting", CASES)
def test_fused_matches_unfused(xse, dtype, dim, tables, batch, combine,
                               weighting):
  rng = np.random.default_rng(dim * 100 + tables * 10 + batch)
  eng, hosts, reqs, meta = build(xse, rng, dtype, dim, tables, batch, combine,
                                 weighting)
  width = dim + (tables + 1) * tables // 2
  out_stride = width + 3
  dense_host = rng.standard_normal((batch, dim)).astype(np.float32)
  dense = torch.from_numpy(dense_host).cuda()
  pooled, want = unfused(xse, eng, reqs, dense, tables, dim, out_stride)
  for t in range(tables):
    ids, offsets, w = meta[t]
    assert_bitwise(pooled[:, t, :],
                   oracle_pool(hosts[t], dtype, ids, offsets, w, combine),
                   f"unfused pooled table {t}")
  out = torch.full((batch, out_stride), 5.0, device="cuda")
  eng.execute_interaction(reqs, dense, out)
  got = out.cpu().numpy()
  np.testing.assert_array_equal(got[:, :dim], dense_host)
  assert np.all(got[:, width:] == 0.0)
  z = np.concatenate([dense_host[:, None, :], pooled], axis=1).astype(
      np.float64)
  mag = np.abs(z) @ np.abs(z).transpose(0, 2, 1)
  iu = np.triu_indices(tables + 1, 1)
  bound = mag[:, iu[0], iu[1]]
  np.testing.assert_array_less(np.abs(got[:, dim:width] - want[:, dim:width]),
                               1e-5 * bound + 1e-12)
  np.testing.assert_array_less(
      np.abs(got[:, dim:width] - oracle.dot_interaction(
          dense_host, pooled)[:, dim:]), 1e-4 * bound + 1e-7)

  # One-hot dense rows: pair (0, 1 + t) is pooled[b, t, c_b] (hi + lo).
  cols = rng.integers(0, dim, batch)
  onehot = np.zeros((batch, dim), np.float32)
  onehot[np.arange(batch), cols] = 1.0
  eng.execute_interaction(reqs, torch.from_numpy(onehot).cuda(), out)
  got = out.cpu().numpy()[:, dim:dim + tables].astype(np.float64)
  want_rows = pooled[np.arange(batch), :, cols].astype(np.float64)
  np.testing.assert_array_less(np.abs(got - want_rows),
                               2.0 ** -20 * np.abs(want_rows) + 1e-30)
  eng.close()


def test_fused_async_strict_and_errors(xse):
  """Strict and fused checks report the pooled lookup's errors with the same
  messages as execute_batch; shape errors are caught before any launch."""
  rng = np.random.default_rng(3)
  eng, _, reqs, meta = build(xse, rng, oracle.F32, 128, 4, 16, "SUM", None)
  dense = torch.randn(16, 128, device="cuda")
  width = 128 + 10
  out = torch.zeros((16, width), device="cuda")
  st = xse.Status(8)
  eng.execute_interaction(reqs, dense, out, status=st)
  st.wait()
  ids, offsets, _ = meta[2]
  bad = ids.copy()
  pos = int(offsets[5])
  bad[pos] = 10 ** 6
  bad_reqs = list(reqs)
  bad_reqs[2] = xse.BagRequest("f2", to_dev(bad), to_dev(offsets), None)
  for fused in (False, True):
    before = out.clone()
    with pytest.raises(xse.XseError) as e:
      eng.execute_interaction(bad_reqs, dense, out, fused=fused)
    assert e.value.message == (
        f"FP32 embedding-bag request 2: Embedding ID ({10 ** 6}) at index "
        f"{pos} is out of bounds [0, {eng.table_info('t2').vocab}).")
    if not fused:  # strict: the kernel did not run
      assert torch.equal(out, before)
  short = [xse.BagRequest(r.feature_name, r.ids, r.offsets[:-1], None)
           for r in reqs]
  with pytest.raises(xse.XseError) as e:
    eng.execute_interaction(short, dense, out)
  assert e.value.message == (
      "Interaction request 0 has 15 bags; the batch has 16 samples.")
  with pytest.raises(xse.XseError) as e:
    eng.execute_interaction(reqs, dense,
                            torch.zeros((16, width - 1), device="cuda"))
  assert "Interaction strides too small" in e.value.message
  eng.add_table("narrow", torch.zeros((10, 64), device="cuda"), "SUM")
  eng.register_feature("fn", "narrow")
  mixed = reqs[:3] + [xse.BagRequest("fn", reqs[3].ids[:0].clone(),
                                     torch.zeros(17, dtype=torch.int64,
                                                 device="cuda"), None)]
  with pytest.raises(xse.XseError) as e:
    eng.execute_interaction(mixed, dense, out)
  assert e.value.message == (
      "Interaction request 3 has dimension 64; request 0 has 128.")
  st.close()
  eng.close()
