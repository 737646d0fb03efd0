"""GPU tests of the CSR packing kernels (include/xse_shard.h) behind the ids
all-to-all of table-wise sharding: extents and packed ids, weights and
rebased offsets compared element for element with the same slices taken on
the host; bad ranges reported as -1 and skipped. Then a one-rank
IdsAllToAll + TablewiseExchange round (no collective at world size 1) is
checked bit for bit against pooling the whole batch directly."""

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import assert_bitwise, random_table, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sharding(xse):
  return xse.sharding


@pytest.mark.parametrize("id_dtype", [torch.int64, torch.int32])
def test_pack_matches_host_slices(xse, sharding, id_dtype):
  rng = np.random.default_rng(9)
  jobs_src, want = [], []
  for k in range(7):
    bags = int(rng.integers(1, 300))
    lengths = rng.integers(0, 9, bags)
    first = int(rng.integers(0, 5))
    offsets = np.concatenate([[first], first + np.cumsum(lengths)])
    ids = rng.integers(-5, 1000, int(offsets[-1]) + int(rng.integers(0, 4)))
    weights = (rng.uniform(0, 1, len(ids)).astype(np.float32)
               if k % 2 else None)
    off_t = torch.from_numpy(offsets.astype(np.int64 if k % 3 else np.int32))
    jobs_src.append((to_dev(ids, id_dtype), off_t.cuda(),
                     None if weights is None else to_dev(weights)))
    want.append((ids[offsets[0]:offsets[-1]], offsets - offsets[0],
                 None if weights is None else weights[offsets[0]:offsets[-1]]))
  packer = sharding.CsrPacker()
  ext = packer.extents([j + (None, None, None, 0) for j in jobs_src]).cpu()
  assert ext.tolist() == [len(w[0]) for w in want]
  total = int(ext.sum())
  dst_ids = torch.full((total,), -99, dtype=id_dtype, device="cuda")
  dst_w = torch.full((total,), -1.0, device="cuda")
  dst_offs = [torch.empty(len(w[1]), dtype=torch.int64, device="cuda")
              for w in want]
  jobs, at = [], 0
  for (ids, offs, w), d_offs, n in zip(jobs_src, dst_offs, ext.tolist()):
    jobs.append((ids, offs, w, dst_ids[at:at + n], d_offs, dst_w[at:at + n],
                 at))
    at += n
  packer.pack(jobs)
  got_ids, got_w = dst_ids.cpu().numpy(), dst_w.cpu().numpy()
  at = 0
  for (ids, offs, w), d_offs in zip(want, dst_offs):
    n = len(ids)
    np.testing.assert_array_equal(got_ids[at:at + n], ids)
    np.testing.assert_array_equal(d_offs.cpu().numpy(), offs + at)
    if w is None:
      assert np.all(got_w[at:at + n] == -1.0)
    else:
      np.testing.assert_array_equal(got_w[at:at + n], w)
    at += n


def test_bad_ranges(xse, sharding):
  ids = to_dev(np.arange(10))
  bad = [torch.tensor(o, dtype=torch.int64, device="cuda") for o in
         ([-1, 3], [4, 2], [2, 11], [0, 10], [10, 10])]
  packer = sharding.CsrPacker()
  ext = packer.extents([(ids, o, None, None, None, None, 0) for o in bad])
  assert ext.cpu().tolist() == [-1, -1, -1, 10, 0]
  d_offs = torch.full((2,), 7, dtype=torch.int64, device="cuda")
  packer.pack([(ids, bad[0], None, ids[:0].clone(), d_offs, None, 0)])
  assert d_offs.cpu().tolist() == [7, 7]  # skipped
  C = xse._capi
  assert C.lib.xse_csr_pack(None, 1, None) == C.INVALID_ARGUMENT


def test_one_rank_round_matches_direct_pooling(xse, sharding):
  rng = np.random.default_rng(4)
  eng = xse.EmbeddingEngine(0)
  plan = sharding.ShardPlan(1, 0)
  batch, dim, tables = 96, 32, 3
  dp, hosts, whole = [], [], []
  for t in range(tables):
    host, dev, _, _ = random_table(rng, oracle.F32, 200, dim)
    eng.add_table(f"t{t}", dev, "MEAN" if t == 1 else "SUM")
    eng.register_feature(f"f{t}", f"t{t}")
    lengths = rng.integers(0, 7, batch)
    offsets = np.concatenate([[3], 3 + np.cumsum(lengths)])
    ids = rng.integers(0, 200, int(offsets[-1]))
    w = rng.uniform(0, 1, len(ids)).astype(np.float32) if t == 2 else None
    dp.append((f"f{t}", to_dev(ids), to_dev(offsets),
               None if w is None else to_dev(w)))
    whole.append(oracle.embedding_bag(host, ids, offsets, w,
                                      "MEAN" if t == 1 else "SUM"))
  ids_a2a = sharding.IdsAllToAll(plan, batch, tables)
  ex = sharding.TablewiseExchange(plan, batch, tables, dim,
                                  sharding.engine_pooler(eng), device="cuda")
  blocks = ids_a2a.run(dp)
  ex.run(ex.schedule(blocks=blocks))
  got = ex.sample_major().cpu().numpy()
  for t in range(tables):
    assert_bitwise(got[:, t, :], whole[t], f"table {t}")
  eng.close()
