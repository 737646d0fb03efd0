"""Sharded execution through the C ABI (include/xse_shard.h):
xse_shard_comm_* and xse_shard_exchange_* in every mode -- table-wise with
peer stores, one all-to-all, or the pipelined send/recv, and row-wise
windows with the chunked reduce-scatter.

On one GPU the job has one rank (a one-rank NCCL communicator; every mode
reduces to pooling into the output layout). On two GPUs (one process each)
every rank's output [B/W, T, D] -- its samples of every table,
sample-major -- is compared with the oracle pooling every table over the
whole batch: bit for bit table-wise, within 1e-5 of the magnitude sum
row-wise (partials are added in another order). The exchange's own request
checks are exercised too."""

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

NUM_TABLES, VOCAB, DIM, BATCH = 6, 2999, 128, 512
COMBINE = ["SUM", "MEAN", "SQRT_N", "SUM", "MEAN", "SUM"]
MODES = ["peer", "a2a", "pipelined", "row"]


def table_bits(t):
  return oracle.synth_rows(oracle.BF16, 9, t, 0, VOCAB, DIM)[0]


def batch_of(t, step=0):
  rng = np.random.default_rng(700 + 31 * t + step)
  lengths = rng.integers(0, 35, BATCH)
  offsets = np.concatenate([[2], 2 + np.cumsum(lengths)]).astype(np.int64)
  ids = rng.integers(0, VOCAB, int(offsets[-1])).astype(np.int64)
  ids[:2] = -1  # before the first offset: never read
  weights = rng.uniform(0, 1, len(ids)).astype(np.float32) if t % 2 else None
  return ids, offsets, weights


def full_pooled(step):
  out = np.zeros((BATCH, NUM_TABLES, DIM), np.float32)
  for t in range(NUM_TABLES):
    ids, offsets, weights = batch_of(t, step)
    out[:, t] = oracle.embedding_bag(table_bits(t), ids, offsets, weights,
                                     COMBINE[t], oracle.BF16)
  return out


def run_rank(xse, rank, world, mode, steps=5):
  """Builds this rank's engine and exchange, runs `steps` steps (different
  inputs each) and returns the outputs of every step as numpy arrays."""
  sharding = xse.sharding
  plan = sharding.ShardPlan(world, rank)
  engine = xse.EmbeddingEngine(rank)
  comm = sharding.ShardComm(rank, plan)
  rowwise = mode == "row"
  tables = (range(NUM_TABLES) if rowwise else
            plan.tables_of(rank, NUM_TABLES))
  for t in tables:
    bits = torch.from_numpy(table_bits(t).view(np.int16)).view(torch.bfloat16)
    if rowwise:
      lo, hi = plan.row_window(VOCAB)
      engine.add_table(f"f{t}", bits[lo:hi].cuda(), COMBINE[t], vocab=VOCAB,
                       row_begin=lo, row_end=hi)
    else:
      engine.add_table(f"f{t}", bits.cuda(), COMBINE[t])
    engine.register_feature(f"f{t}", f"f{t}")
  ex = sharding.ShardedExchange(engine, comm, mode, NUM_TABLES, DIM, BATCH,
                                chunks=2 if rowwise else 1)
  outs = []
  keep = []
  for step in range(steps):
    feats = []
    for t in tables:
      ids, offsets, weights = batch_of(t, step)
      feats.append((f"f{t}", torch.from_numpy(ids).cuda(),
                     torch.from_numpy(offsets).cuda(),
                     None if weights is None else
                     torch.from_numpy(weights).cuda()))
    keep.append(feats)
    # Deferred steps (the next step's pooling overlaps this step's exchange)
    # except the last; readers are queued after ready(), before the next
    # run (the slot reuse rule). Five steps rotate the peer mode's three
    # output slots past their first reuse.
    last = step == steps - 1
    out = ex.run(ex.prepare(feats), defer=not last and step % 2 == 0)
    ex.ready()
    outs.append(out.clone())
  ex.check()
  result = [o.cpu().numpy() for o in outs]
  ex.close()
  comm.close()
  engine.close()
  return result


def compare(got, step, rank, world, mode):
  want = full_pooled(step)
  block = BATCH // world
  exp = want[rank * block:(rank + 1) * block]
  if mode == "row" and world > 1:
    np.testing.assert_allclose(got, exp, rtol=1e-5, atol=1e-6)
  else:
    np.testing.assert_array_equal(got.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("mode", MODES)
def test_one_rank_exchange(xse, mode):
  outs = run_rank(xse, 0, 1, mode)
  for step, got in enumerate(outs):
    compare(got, step, 0, 1, mode)


def test_exchange_rejects_bad_requests(xse):
  sharding = xse.sharding
  plan = sharding.ShardPlan(1, 0)
  engine = xse.EmbeddingEngine(0)
  comm = sharding.ShardComm(0, plan)
  bits = torch.from_numpy(table_bits(0).view(np.int16)).view(torch.bfloat16)
  engine.add_table("f0", bits.cuda(), "SUM")
  engine.register_feature("f0", "f0")
  with pytest.raises(xse.XseError) as e:  # batch not divisible: 1 rank ok,
    sharding.ShardedExchange(engine, comm, "peer", 1, 130, 8)  # dim % 4
  assert e.value.code == xse._capi.INVALID_ARGUMENT
  ex = sharding.ShardedExchange(engine, comm, "a2a", 1, DIM, 16)
  ids = torch.zeros(4, dtype=torch.int64, device="cuda")
  with pytest.raises(xse.XseError) as e:  # 5 offsets for a batch of 16
    ex.run([("f0", ids, torch.arange(5, device="cuda"), None)])
  assert "row pointers" in e.value.message
  # An out-of-range id is reported by check() with the engine's message.
  offs = torch.arange(17, device="cuda") // 4
  bad = torch.tensor([0, 1, VOCAB, 3], device="cuda")
  ex.run([("f0", bad, offs, None)])
  with pytest.raises(xse.XseError) as e:
    ex.check()
  assert e.value.message == ("FP32 embedding-bag request 0: Embedding ID "
                             f"({VOCAB}) at index 2 is out of bounds [0, "
                             f"{VOCAB}).")
  ex.close()
  comm.close()
  engine.close()


def _rendezvous():
  """A rendezvous for the ranks of one test: a FileStore in a fresh
  temporary directory (no TCP port that another process could take
  between choosing it and the store binding it)."""
  return "file://" + os.path.join(tempfile.mkdtemp(prefix="xse_rdv_"),
                                  "store")


def _rank_main(rank, world, rendezvous, mode, results):
  os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
  torch.cuda.set_device(rank)
  dist.init_process_group("nccl", init_method=rendezvous, rank=rank,
                          world_size=world,
                          timeout=timedelta(seconds=60),
                          device_id=torch.device("cuda", rank))
  try:
    from conftest import load_package  # pylint: disable=import-outside-toplevel
    xse = load_package()
    results[rank] = run_rank(xse, rank, world, mode)
  finally:
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", MODES)
def test_two_gpu_exchange(mode):
  if torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs")
  world = 2
  with mp.get_context("spawn").Manager() as manager:
    results = manager.dict()
    mp.start_processes(_rank_main, args=(world, _rendezvous(), mode, results),
                       nprocs=world, start_method="spawn")
    got = {r: results[r] for r in range(world)}
  for r in range(world):
    for step, out in enumerate(got[r]):
      compare(out, step, r, world, mode)
