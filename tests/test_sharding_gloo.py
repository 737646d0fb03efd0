"""CPU tests of the sharded paths' host logic with world-size-2 gloo ranks:
placement, sample-block request slicing, the pipelined pairwise exchange,
the chunked reduce-scatter and the ids all-to-all of data-parallel input. Each rank pools with the oracle on the CPU (the
test stands in for the GPU pooling kernels), then the exchanged result is
compared with one process pooling every table over the whole batch: bit for
bit table-wise, within 1e-5 of the magnitude sum row-wise (partial sums are
added in another order)."""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle

NUM_TABLES, VOCAB, DIM, BATCH = 5, 211, 12, 24


def make_tables():
  rng = np.random.default_rng(7)
  return [rng.uniform(-1, 1, (VOCAB, DIM)).astype(np.float32)
          for _ in range(NUM_TABLES)]


def make_batch(t):
  rng = np.random.default_rng(100 + t)
  lengths = rng.integers(0, 6, BATCH)
  offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
  ids = rng.integers(0, VOCAB, int(offsets[-1])).astype(np.int64)
  weights = rng.uniform(0, 1, len(ids)).astype(np.float32) if t % 2 else None
  return ids, offsets, weights


COMBINE = ["SUM", "MEAN", "SQRT_N", "SUM", "MEAN"]


def cpu_pooler(tables_by_feature):
  """Pools bag requests of CPU tensors with the oracle, writing each
  request's (strided) output view."""
  def pool(reqs):
    for r in reqs:
      table, combine = tables_by_feature[r.feature_name]
      w = None if r.weights is None else r.weights.numpy()
      out = oracle.embedding_bag(table, r.ids.numpy(), r.offsets.numpy(), w,
                                 combine)
      r.output.copy_(torch.from_numpy(out))
  return pool


def full_pooled(tables):
  out = np.zeros((BATCH, NUM_TABLES, DIM), np.float32)
  for t in range(NUM_TABLES):
    ids, offsets, weights = make_batch(t)
    out[:, t] = oracle.embedding_bag(tables[t], ids, offsets, weights,
                                     COMBINE[t])
  return out


def _rendezvous():
  """A rendezvous for the ranks of one test: a FileStore in a fresh
  temporary directory (no TCP port that another process could take
  between choosing it and the store binding it)."""
  return "file://" + os.path.join(tempfile.mkdtemp(prefix="xse_rdv_"),
                                  "store")


def _tablewise_rank(rank, world, rendezvous, mode, results):
  dist.init_process_group("gloo", init_method=rendezvous, rank=rank,
                          world_size=world)
  try:
    from conftest import load_package  # pylint: disable=import-outside-toplevel
    sharding = load_package().sharding
    plan = sharding.ShardPlan(world, rank)
    tables = make_tables()
    local = plan.tables_of(rank, NUM_TABLES)
    features, by_name = [], {}
    for t in local:
      ids, offsets, weights = make_batch(t)
      name = f"f{t}"
      by_name[name] = (tables[t], COMBINE[t])
      features.append((name, torch.from_numpy(ids), torch.from_numpy(offsets),
                       None if weights is None else torch.from_numpy(weights)))
    ex = sharding.TablewiseExchange(plan, BATCH, NUM_TABLES, DIM,
                                    cpu_pooler(by_name), mode=mode)
    ex.send.fill_(float("nan"))
    ex.recv.fill_(float("nan"))
    ex.run(ex.schedule(features))
    results[rank] = ex.sample_major().numpy().copy()
  finally:
    dist.destroy_process_group()


class TorchPacker:
  """The packing step of sharding.IdsAllToAll on CPU tensors (the GPU runs
  the kernels of include/xse_shard.h; this stands in for them here)."""

  @staticmethod
  def extents(jobs):
    out = []
    for ids, offsets, _, *_ in jobs:
      lo, hi = int(offsets[0]), int(offsets[-1])
      out.append(hi - lo if 0 <= lo <= hi <= ids.numel() else -1)
    return torch.tensor(out, dtype=torch.int64)

  @staticmethod
  def pack(jobs):
    for ids, offsets, weights, d_ids, d_offs, d_w, base in jobs:
      lo, hi = int(offsets[0]), int(offsets[-1])
      d_ids.copy_(ids[lo:hi])
      d_offs.copy_(offsets.to(torch.int64) - lo + base)
      if weights is not None and d_w is not None:
        d_w.copy_(weights[lo:hi])


def _ids_a2a_rank(rank, world, rendezvous, mode, results):
  """Data-parallel input: this rank holds every table's ids for its own
  sample block only (absolute offsets into the whole batch's arrays)."""
  dist.init_process_group("gloo", init_method=rendezvous, rank=rank,
                          world_size=world)
  try:
    from conftest import load_package  # pylint: disable=import-outside-toplevel
    sharding = load_package().sharding
    plan = sharding.ShardPlan(world, rank)
    tables = make_tables()
    b0, b1 = plan.sample_block(BATCH, rank)
    dp, by_name = [], {}
    for t in range(NUM_TABLES):
      ids, offsets, weights = make_batch(t)
      name = f"f{t}"
      by_name[name] = (tables[t], COMBINE[t])
      dp.append((name, torch.from_numpy(ids),
                 torch.from_numpy(offsets[b0:b1 + 1]),
                 None if weights is None else torch.from_numpy(weights)))
    ids_a2a = sharding.IdsAllToAll(plan, BATCH, NUM_TABLES,
                                   packer=TorchPacker())
    ex = sharding.TablewiseExchange(plan, BATCH, NUM_TABLES, DIM,
                                    cpu_pooler(by_name), mode=mode)
    ex.recv.fill_(float("nan"))
    for _ in range(2):  # buffers are rebuilt per step
      blocks = ids_a2a.run(dp)
      ex.run(ex.schedule(blocks=blocks))
    results[rank] = ex.sample_major().numpy().copy()
  finally:
    dist.destroy_process_group()


def _rowwise_rank(rank, world, rendezvous, chunks, results):
  dist.init_process_group("gloo", init_method=rendezvous, rank=rank,
                          world_size=world)
  try:
    from conftest import load_package  # pylint: disable=import-outside-toplevel
    sharding = load_package().sharding
    plan = sharding.ShardPlan(world, rank)
    tables = make_tables()
    features, by_name = [], {}
    for t in range(NUM_TABLES):
      lo, hi = plan.row_window(VOCAB)
      shard = np.zeros_like(tables[t])  # rows of other shards contribute 0
      shard[lo:hi] = tables[t][lo:hi]
      ids, offsets, weights = make_batch(t)
      name = f"f{t}"
      by_name[name] = (shard, COMBINE[t])
      features.append((name, torch.from_numpy(ids), torch.from_numpy(offsets),
                       None if weights is None else torch.from_numpy(weights)))
    ex = sharding.RowwiseExchange(plan, BATCH, NUM_TABLES, DIM,
                                  cpu_pooler(by_name), chunks=chunks)
    recv = ex.run(ex.schedule(features))
    results[rank] = recv.numpy().copy()
  finally:
    dist.destroy_process_group()


def _spawn(fn, *args):
  world = 2
  with mp.get_context("spawn").Manager() as manager:
    results = manager.dict()
    mp.start_processes(fn, args=(world, _rendezvous()) + args + (results,),
                       nprocs=world, start_method="spawn")
    return [results[r] for r in range(world)]


def test_shard_plan():
  from conftest import load_package  # pylint: disable=import-outside-toplevel
  sharding = load_package().sharding
  plan = sharding.ShardPlan(4, 1)
  assert plan.tables_of(1, 10) == [1, 5, 9]
  assert [plan.table_owner(t) for t in range(6)] == [0, 1, 2, 3, 0, 1]
  windows = [plan.row_window(10, r) for r in range(4)]
  assert windows == [(0, 2), (2, 5), (5, 7), (7, 10)]
  assert plan.sample_block(64, 3) == (48, 64)
  with pytest.raises(ValueError):
    plan.block_size(30)
  with pytest.raises(ValueError):
    sharding.ShardPlan(2, 2)


def test_slice_request_keeps_absolute_offsets():
  from conftest import load_package  # pylint: disable=import-outside-toplevel
  xse = load_package()
  ids = torch.arange(10)
  offsets = torch.tensor([0, 2, 5, 5, 9, 10])
  out = torch.empty(2, 3)
  base = xse.BagRequest("f", ids, offsets, None)
  r = xse.sharding.slice_request(base, 2, 4, out)
  assert r.offsets.tolist() == [5, 5, 9] and r.ids is ids and r.output is out


@pytest.mark.parametrize("mode", ["pipelined", "a2a"])
def test_tablewise_exchange_gloo(mode):
  tables = make_tables()
  want = full_pooled(tables)
  got = _spawn(_tablewise_rank, mode)
  world = 2
  block = BATCH // world
  for r in range(world):
    np.testing.assert_array_equal(got[r], want[r * block:(r + 1) * block])


@pytest.mark.parametrize("mode", ["pipelined", "a2a"])
def test_ids_all_to_all_then_tablewise_gloo(mode):
  """Data-parallel ids moved to the table owners (IdsAllToAll), pooled there
  and returned: the same rows, bit for bit, as pooling every table over the
  whole batch in one process."""
  tables = make_tables()
  want = full_pooled(tables)
  got = _spawn(_ids_a2a_rank, mode)
  world = 2
  block = BATCH // world
  for r in range(world):
    np.testing.assert_array_equal(got[r], want[r * block:(r + 1) * block])


@pytest.mark.parametrize("chunks", [1, 3])
def test_rowwise_reduce_scatter_gloo(chunks):
  tables = make_tables()
  want = full_pooled(tables)
  got = _spawn(_rowwise_rank, chunks)
  world = 2
  block = BATCH // world
  for r in range(world):
    exp = want[r * block:(r + 1) * block]
    np.testing.assert_allclose(got[r], exp, rtol=1e-5, atol=1e-6)


def _leaving_rank(rank, world, rendezvous, mode, results):
  """Both ranks run one exchange step; then rank 1 leaves (between steps,
  nothing of it in flight) and rank 0 runs the next step. Rank 0's
  collective must end with an error within the process group's short
  timeout instead of waiting for ever."""
  import time  # pylint: disable=import-outside-toplevel
  from datetime import timedelta  # pylint: disable=import-outside-toplevel
  dist.init_process_group("gloo", init_method=rendezvous, rank=rank,
                          world_size=world,
                          timeout=timedelta(seconds=5))
  try:
    from conftest import load_package  # pylint: disable=import-outside-toplevel
    sharding = load_package().sharding
    plan = sharding.ShardPlan(world, rank)
    tables = make_tables()
    rowwise = mode == "rowwise"
    local = (range(NUM_TABLES) if rowwise
             else plan.tables_of(rank, NUM_TABLES))
    features, by_name = [], {}
    for t in local:
      ids, offsets, weights = make_batch(t)
      by_name[f"f{t}"] = (tables[t], COMBINE[t])
      features.append((f"f{t}", torch.from_numpy(ids),
                       torch.from_numpy(offsets),
                       None if weights is None else torch.from_numpy(weights)))
    if rowwise:
      ex = sharding.RowwiseExchange(plan, BATCH, NUM_TABLES, DIM,
                                    cpu_pooler(by_name), chunks=2)
    else:
      ex = sharding.TablewiseExchange(plan, BATCH, NUM_TABLES, DIM,
                                      cpu_pooler(by_name), mode=mode)
    steps = ex.schedule(features)
    ex.run(steps)  # every rank takes part
    if rank == 1:
      results[1] = "left"
      return
    t0 = time.monotonic()
    try:
      ex.run(steps)
      results[0] = ("no error", time.monotonic() - t0)
    except Exception as e:  # pylint: disable=broad-except
      results[0] = (type(e).__name__, time.monotonic() - t0)
  finally:
    try:
      dist.destroy_process_group()
    except Exception:  # pylint: disable=broad-except
      pass


@pytest.mark.parametrize("mode", ["a2a", "pipelined", "rowwise"])
def test_rank_leaving_between_steps_ends_the_next_exchange(mode):
  got = _spawn(_leaving_rank, mode)
  assert got[1] == "left"
  kind, seconds = got[0]
  assert kind != "no error", got[0]
  assert seconds < 60, got[0]
