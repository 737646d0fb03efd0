"""Sharded pooling on two GPUs (one process each, NCCL): table-wise placement
with the pipelined pairwise exchange, with one all-to-all and with pooled rows
stored straight into the owner's buffer over NVLink, and row-wise windows
with the chunked reduce-scatter, and data-parallel input moved to the table
owners by the ids all-to-all, through the engine's kernels. The
result on each rank is compared with the oracle pooling every table over the
whole batch: bit for bit table-wise, within 1e-5 relative to the magnitude
sum row-wise (partials are added in another order). Needs two GPUs."""

import os
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle

pytestmark = pytest.mark.gpu

NUM_TABLES, VOCAB, DIM, BATCH = 5, 3001, 128, 256
COMBINE = ["SUM", "MEAN", "SQRT_N", "SUM", "MEAN"]


def table_bits(t):
  return oracle.synth_rows(oracle.BF16, 5, t, 0, VOCAB, DIM)[0]


def batch_of(t):
  rng = np.random.default_rng(300 + t)
  lengths = rng.integers(0, 40, BATCH)
  offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
  ids = rng.integers(0, VOCAB, int(offsets[-1])).astype(np.int64)
  weights = rng.uniform(0, 1, len(ids)).astype(np.float32) if t % 2 else None
  return ids, offsets, weights


def _rendezvous():
  """A rendezvous for the ranks of one test: a FileStore in a fresh
  temporary directory (no TCP port that another process could take
  between choosing it and the store binding it)."""
  return "file://" + os.path.join(tempfile.mkdtemp(prefix="xse_rdv_"),
                                  "store")


def _rank_main(rank, world, rendezvous, mode, results):
  torch.cuda.set_device(rank)
  dist.init_process_group("nccl", init_method=rendezvous, rank=rank,
                          world_size=world,
                          timeout=timedelta(seconds=60),
                          device_id=torch.device("cuda", rank))
  try:
    from conftest import load_package  # pylint: disable=import-outside-toplevel
    xse = load_package()
    sharding = xse.sharding
    plan = sharding.ShardPlan(world, rank)
    engine = xse.EmbeddingEngine(rank)
    status = xse.Status(NUM_TABLES * world)
    pool = sharding.engine_pooler(engine, status)
    features = []
    tables = (range(NUM_TABLES) if mode == "rowwise"
              else plan.tables_of(rank, NUM_TABLES))
    for t in tables:
      bits = torch.from_numpy(table_bits(t).view(np.int16)).view(
          torch.bfloat16)
      name = f"f{t}"
      if mode == "rowwise":
        lo, hi = plan.row_window(VOCAB)
        engine.add_table(name, bits[lo:hi].cuda(), COMBINE[t], vocab=VOCAB,
                         row_begin=lo, row_end=hi)
      else:
        engine.add_table(name, bits.cuda(), COMBINE[t])
      engine.register_feature(name, name)
      ids, offsets, weights = batch_of(t)
      features.append((name, torch.from_numpy(ids).cuda(),
                       torch.from_numpy(offsets).cuda(),
                       None if weights is None else
                       torch.from_numpy(weights).cuda()))
    if mode.startswith("ids_a2a"):
      # Data-parallel input: every table's ids for this rank's samples only.
      b0, b1 = plan.sample_block(BATCH, rank)
      dp = []
      for t in range(NUM_TABLES):
        ids, offsets, weights = batch_of(t)
        dp.append((f"f{t}", torch.from_numpy(ids).cuda(),
                   torch.from_numpy(offsets[b0:b1 + 1]).cuda(),
                   None if weights is None else
                   torch.from_numpy(weights).cuda()))
      ids_a2a = sharding.IdsAllToAll(plan, BATCH, NUM_TABLES, device="cuda")
      ex = sharding.TablewiseExchange(plan, BATCH, NUM_TABLES, DIM, pool,
                                      device="cuda",
                                      mode=mode.split("_")[2])
      outs = []
      for _ in range(3):
        ex.run(ex.schedule(blocks=ids_a2a.run(dp)))
        outs.append(ex.sample_major())
      status.wait()
      ex.check()
      for o in outs[:-1]:
        torch.testing.assert_close(o, outs[-1], rtol=0, atol=0)
      out = outs[-1]
      ex.close()
    elif mode == "rowwise":
      ex = sharding.RowwiseExchange(plan, BATCH, NUM_TABLES, DIM, pool,
                                    chunks=2, device="cuda")
      for _ in range(2):  # twice: buffers are reused across steps
        out = ex.run(ex.schedule(features))
      status.wait()
    else:
      ex = sharding.TablewiseExchange(plan, BATCH, NUM_TABLES, DIM, pool,
                                      device="cuda",
                                      mode=mode.split("_")[1])
      steps = ex.schedule(features)
      outs = []
      for _ in range(3):  # peer mode alternates receive slots
        ex.run(steps)
        outs.append(ex.sample_major())
      status.wait()
      ex.check()
      for o in outs[:-1]:
        torch.testing.assert_close(o, outs[-1], rtol=0, atol=0)
      out = outs[-1]
      ex.close()
    torch.cuda.synchronize()
    results[rank] = out.cpu().numpy()
    status.close()
    engine.close()
  finally:
    dist.destroy_process_group()


def full_pooled():
  out = np.zeros((BATCH, NUM_TABLES, DIM), np.float32)
  for t in range(NUM_TABLES):
    ids, offsets, weights = batch_of(t)
    out[:, t] = oracle.embedding_bag(table_bits(t), ids, offsets, weights,
                                     COMBINE[t], oracle.BF16)
  return out


@pytest.mark.parametrize("mode", ["tablewise_pipelined", "tablewise_a2a",
                                  "tablewise_peer", "rowwise",
                                  "ids_a2a_peer", "ids_a2a_pipelined"])
def test_sharded_two_gpus(mode):
  if torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs")
  world = 2
  with mp.get_context("spawn").Manager() as manager:
    results = manager.dict()
    mp.start_processes(_rank_main, args=(world, _rendezvous(), mode, results),
                       nprocs=world, start_method="spawn")
    got = [results[r] for r in range(world)]
  want = full_pooled()
  block = BATCH // world
  for r in range(world):
    exp = want[r * block:(r + 1) * block]
    if mode == "rowwise":
      np.testing.assert_allclose(got[r], exp, rtol=1e-5, atol=1e-6)
    else:
      np.testing.assert_array_equal(got[r], exp)


def _barrier_timeout_main(rank, world, rendezvous, results):
  """Rank 1 never reaches the barrier: rank 0's bounded wait gives up and
  the group reports DEADLINE_EXCEEDED; the context stays usable."""
  torch.cuda.set_device(rank)
  dist.init_process_group("nccl", init_method=rendezvous, rank=rank,
                          world_size=world,
                          timeout=timedelta(seconds=60),
                          device_id=torch.device("cuda", rank))
  try:
    from conftest import load_package  # pylint: disable=import-outside-toplevel
    xse = load_package()
    plan = xse.sharding.ShardPlan(world, rank)
    group = xse.sharding.PeerGroup(plan, 1024, rank)
    group.barrier()  # both ranks: passes
    group.check()
    if rank == 0:
      group.barrier(spin_limit=2000)  # rank 1 never comes: ~ms, then gives up
      try:
        group.check()
        results[rank] = "no error"
      except xse.XseError as e:
        results[rank] = (e.code, e.message)
      x = torch.ones(4, device="cuda")
      results["usable"] = float((x * 2).sum().item())
    dist.barrier()
    group.close()
  finally:
    dist.destroy_process_group()


def test_peer_barrier_gives_up_when_a_rank_never_arrives(xse):
  if torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs")
  with mp.get_context("spawn").Manager() as manager:
    results = manager.dict()
    mp.start_processes(_barrier_timeout_main,
                       args=(2, _rendezvous(), results), nprocs=2,
                       start_method="spawn")
    got = dict(results)
  assert got[0][0] == xse._capi.DEADLINE_EXCEEDED
  assert "gave up" in got[0][1]
  assert got["usable"] == 8.0
