#!/usr/bin/env python3
"""Benchmark of the B200 embedding-bag engine.

Headline workload (one GPU): multi-table weighted/mean pooling -- 8 bf16
tables of 500,000 x 128 rows, batch 8192, 20 ids per bag, uniform ids, per-id
fp32 weights U(0,1); tables 0-3 pool as weighted sums, 4-7 as means; fp32
accumulation; output 8192 x 8 x 128 fp32. A step is one pooled lookup of one
batch over all tables (one execute_batch group: a validation kernel and a
pooling kernel).

With N GPUs (torchrun, one process per GPU, NCCL) every rank holds 8 such
tables (8N tables in all, table-wise sharded) and pools them for the whole
batch; each sample block goes to its owning rank (weak scaling: fixed work
per GPU). By default the pooling kernel stores the blocks straight into the
owners' buffers over NVLink and a flag barrier ends the step (--exchange
peer); --exchange a2a / pipelined use NCCL instead.

The same run measures the other workloads and reports each under its own key
of the one JSON line (each with its roofline, end-to-end rate, CPU baseline
and parity check at N=1):
  zipf_single        1 fp32 table 1M x 64, batch 4096, U[1,32], Zipf(1.05)
  sharded_tablewise  64 bf16 tables 20M x 128, 8 per GPU, batch 65536,
                     U[1,64], Zipf(1.1), table-wise exchange
  int8_rowwise       26 int8 tables 10M x 256, row-wise windows over the N
                     GPUs, batch 32768, U[1,80], Zipf(1.05), reduce-scatter
  dlrm_forward       DLRM forward, 26 fp32 tables x 128, batch 16384
  dlrm_lookup        the reference's own DLRM bundle lookup: 26 fp32 tables
                     of its vocabulary sizes, valencies 1-100 (214 ids per
                     example), uniform int32 [B, valency] ids through
                     CpuEmbeddingLookupTransform(dense_lookup=True)

Timing: W untimed warm-up steps, then K steps between CUDA events on the
launching stream (max over ranks), with a barrier and a device synchronize on
both sides. The pooling kernel's own duration comes from a separate pass
after the timed region that records CUDA events around the pooling launch of
every step (at least 16 launches), so no event sits inside the timed steps.

Prints one JSON line (rank 0). `--impl reference` times the CPU restatement
of the reference's embedding-bag (the reference itself cannot be built here)
on the host cores, on the same seeded inputs.
"""

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
PACKAGE_DIR = os.path.join(ROOT, "xla-serving_b200")

# Headline workload constants.
NUM_TABLES = 8
VOCAB = 500_000
DIM = 128
BATCH = 8192
BAG = 20
SEED = 0
ROTATE = 8  # distinct input/output sets cycled between steps (> L2 in all)
E2E_THREADS = 2  # concurrent host callers of the operator in the e2e run
# A config's operator e2e run times about this long (calls sized from a
# warm-up run), so that starting the caller threads stays a small share.
E2E_TARGET_MS = 100.0
MIN_WARMUP = 3
# Pooling launches timed with CUDA events in the kernel-timing pass.
KERNEL_TIMING_LAUNCHES = 24
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one step's
# pooling kernel on one GPU, from the ncu capture of this workload recorded
# with the profiles (reported as `traffic` at N=1 only).
POOL_DRAM_BYTES_PER_STEP = 330.32e6
ROW_BYTES = DIM * 2
WORKLOAD = ("multi_table_bf16: 8 bf16 tables x 500,000 x 128 per GPU, batch "
            "8192, 20 ids per bag, uniform ids, tables 0-3 per-id weighted "
            "sum, 4-7 mean, fp32 accumulate, output 8192x8x128 fp32")
DATA = ("synthetic (seeded counter RNG: uniform ids, U(0,1) weights, "
        "U(-0.05,0.05) rows)")


def load_package():
  name = "xla_serving_b200"
  if name in sys.modules:
    return sys.modules[name]
  spec = importlib.util.spec_from_file_location(
      name, os.path.join(PACKAGE_DIR, "__init__.py"),
      submodule_search_locations=[PACKAGE_DIR])
  module = importlib.util.module_from_spec(spec)
  sys.modules[name] = module
  spec.loader.exec_module(module)
  return module


def load_oracle():
  """The CPU oracle: only the CPU-baseline leg (timing and the parity check
  of the outputs) and the reference arm use it."""
  if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
  from oracle import oracle  # pylint: disable=import-outside-toplevel
  return oracle


def algorithmic_bytes_per_step():
  """Bytes one step must move: every id occurrence's row and id, the weights
  of weighted tables, the int64 offsets and the fp32 outputs (no cache
  credit)."""
  nnz = NUM_TABLES * BATCH * BAG
  weighted_ids = (NUM_TABLES // 2) * BATCH * BAG
  return (nnz * (ROW_BYTES + 8) + weighted_ids * 4 +
          (BATCH + 1) * 8 * NUM_TABLES + BATCH * NUM_TABLES * DIM * 4)


def measured_peaks():
  path = os.path.join(ROOT, "MEASURED_PEAKS.json")
  try:
    with open(path, encoding="utf-8") as f:
      p = json.load(f)
    return float(p["hbm_gbs"]), "measured"
  except (OSError, KeyError, ValueError):
    return 6650.0, "fallback"


class ClockSampler:
  """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

  FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,"
            "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
            "clocks_event_reasons.hw_thermal_slowdown,"
            "clocks_event_reasons.sw_thermal_slowdown,"
            "clocks_event_reasons.sw_power_cap")

  def __init__(self, gpu_index):
    self.gpu_index = gpu_index
    self.proc = None
    self.lines = []
    self.thread = None

  def start(self):
    try:
      self.proc = subprocess.Popen(
          ["nvidia-smi", f"--id={self.gpu_index}",
           f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
           "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
          text=True)
    except OSError:
      self.proc = None
      return
    self.thread = threading.Thread(target=self._read, daemon=True)
    self.thread.start()

  def _read(self):
    for line in self.proc.stdout:
      self.lines.append(line.strip())

  def stop(self):
    if self.proc is None:
      return None
    self.proc.terminate()
    try:
      self.proc.wait(timeout=5)
    except subprocess.TimeoutExpired:
      self.proc.kill()
    if self.thread is not None:
      self.thread.join(timeout=2)
    sm, mx, reasons = [], 0.0, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
             "sw_power_cap"]
    for line in self.lines:
      parts = [p.strip() for p in line.split(",")]
      if len(parts) < 9:
        continue
      try:
        sm.append(float(parts[1]))
        mx = max(mx, float(parts[2]))
      except ValueError:
        continue
      for name, flag in zip(names, parts[5:9]):
        if flag.lower() == "active":
          reasons.add(name)
    if not sm:
      return None
    loaded = [s for s in sm if s >= 0.5 * mx] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
            "reasons": sorted(reasons), "samples": len(sm)}


def init_distributed():
  world = int(os.environ.get("WORLD_SIZE", "1"))
  rank = int(os.environ.get("RANK", "0"))
  local = int(os.environ.get("LOCAL_RANK", "0"))
  if world > 1:
    from datetime import timedelta  # pylint: disable=import-outside-toplevel
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
  return world, rank, local


def barrier(world, local):
  if world > 1:
    dist.barrier(device_ids=[local])


def max_over_ranks(value, world):
  if world == 1:
    return value
  t = torch.tensor([value], dtype=torch.float64, device="cuda")
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  return float(t.item())


def min_over_ranks(value, world):
  if world == 1:
    return value
  t = torch.tensor([value], dtype=torch.float64, device="cuda")
  dist.all_reduce(t, op=dist.ReduceOp.MIN)
  return float(t.item())


def sum_over_ranks(value, world):
  if world == 1:
    return value
  t = torch.tensor([value], dtype=torch.float64, device="cuda")
  dist.all_reduce(t, op=dist.ReduceOp.SUM)
  return float(t.item())


def align_streams(world):
  """Lines the ranks' streams up before a timed region: a one-element NCCL
  all-reduce ends on every GPU at about the same moment, so the start events
  recorded right after it fire together (after a host barrier the ranks'
  host threads wake up tens to hundreds of microseconds apart, and a rank
  that starts early waits for the others inside its timed steps)."""
  if world > 1:
    t = torch.zeros(1, device="cuda")
    dist.all_reduce(t)


def timed_steps(step, first, count, world, local, finish=None):
  """`count` steps between CUDA events on the current stream, with a barrier
  and a synchronize on both sides; returns (max-over-ranks ms, launches)."""
  torch.cuda.synchronize()
  barrier(world, local)
  torch.cuda.synchronize()
  align_streams(world)
  stream = torch.cuda.current_stream()
  start = torch.cuda.Event(enable_timing=True)
  end = torch.cuda.Event(enable_timing=True)
  launches = 0
  start.record(stream)
  for i in range(first, first + count):
    r = step(i)
    launches += r if isinstance(r, int) else 0
  if finish is not None:
    finish()
  end.record(stream)
  torch.cuda.synchronize()
  barrier(world, local)
  return max_over_ranks(start.elapsed_time(end), world), launches


def kernel_timing(engine, step, first, count, finish=None):
  """The pooling kernel's duration: CUDA events around the pooling launch of
  each of `count` further steps (engine profiling, period 1), with another
  event before the validation launch. Returns (mean pooling ms per timed
  launch, timed launches, validation ms per step or None)."""
  torch.cuda.synchronize()
  engine.profile_read()  # restart the sampling
  engine.set_profiling(True, 1)
  for i in range(first, first + count):
    step(i)
  if finish is not None:
    finish()
  torch.cuda.synchronize()
  r = engine.profile_read_stages()
  engine.set_profiling(False)
  n = r["executions"]
  val = r["validate_ms"] / count if r["validated"] else None
  return r["pool_ms"] / max(n, 1), n, val


def validation_share(val_ms, step_ms):
  """The validation kernels' own event-timed duration per step and that
  time against the untimed step (programmatic dependent launch overlaps
  most of it with the previous step's pooling, so the share of the step it
  actually costs is smaller)."""
  if val_ms is None:
    return None
  return {"ms_per_step": val_ms, "fraction_of_step": val_ms / step_ms,
          "timing": "CUDA events before the validation and before the "
                    "pooling launch of each kernel-timing step (kernels "
                    "serialised)"}


def check_parity(items, count, seed=SEED):
  """Part of the CPU-baseline leg: the engine's pooled rows of sampled bags
  (all bags when `count` covers the batch) against the oracle, with the
  touched rows regenerated from the counter RNG on the host. items: dicts
  (dtype, stream, dim, combine, ids, offsets, weights, window, output) per
  table; output is the device [B, dim] view of that table's rows."""
  oracle = load_oracle()
  t0 = time.perf_counter()
  cores = oracle.host_cores()
  summary = {"tables": len(items), "bags_checked": 0, "ok": True,
             "bit_exact": True, "max_abs_err": 0.0, "max_rel_err": 0.0,
             "mismatched": 0}
  rules = set()
  for k, it in enumerate(items):
    offsets = np.asarray(it["offsets"], dtype=np.int64)
    nb = len(offsets) - 1
    bags = oracle.sampled_bags(nb, count, seed + 7919 * k,
                               lengths=np.diff(offsets))
    want, bound = oracle.pool_sampled(
        it["dtype"], SEED, it["stream"], it["dim"], it["combine"], it["ids"],
        offsets, it["weights"], bags, it.get("window"), num_threads=cores)
    idx = torch.from_numpy(bags).to(it["output"].device)
    got = it["output"][idx].cpu().numpy()
    r = oracle.compare_pooled(got, want, bound)
    rules.add(r["rule"])
    summary["bags_checked"] += len(bags)
    summary["ok"] = summary["ok"] and r["ok"]
    summary["bit_exact"] = summary["bit_exact"] and r["bit_exact"]
    summary["mismatched"] += r["mismatched"]
    summary["max_abs_err"] = max(summary["max_abs_err"], r["max_abs_err"])
    summary["max_rel_err"] = max(summary["max_rel_err"], r["max_rel_err"])
  summary["rule"] = " / ".join(sorted(rules))
  summary["seconds"] = time.perf_counter() - t0
  summary["method"] = ("oracle (CPU restatement of ReducePortable/BagScale) "
                       "on the same device-generated ids; rows regenerated "
                       "on the host from the counter RNG")
  return summary


def gather_inputs(feature_sets):
  """Pinned host copies of device tensors (None stays None)."""
  out = []
  for feats in feature_sets:
    out.append([tuple(None if t is None else t.cpu().pin_memory() for t in f)
                for f in feats])
  return out


def tensor_bytes(items):
  return sum(t.numel() * t.element_size() for t in items if t is not None)


# ---------------------------------------------------------------------------
# Headline: multi-table workload.


class Workload:
  """Tables, rotating inputs and outputs of one rank, on its GPU.

  With N ranks the 8N tables are placed table-wise (global table t on rank
  t mod N, so each rank holds 8); each rank pools its tables for the whole
  batch and the exchange returns every sample block to its owner."""

  def __init__(self, xse, rank, world, exchange="peer"):
    from xla_serving_b200 import sharding, synth  # pylint: disable=import-outside-toplevel
    self.xse = xse
    self.world = world
    self.engine = xse.EmbeddingEngine(torch.cuda.current_device())
    self.plan = sharding.ShardPlan(world, rank)
    total = NUM_TABLES * world
    self.global_tables = self.plan.tables_of(rank, total)
    specs = synth.multi_table_specs()
    self.specs = []
    self.tables = []
    for k, g in enumerate(self.global_tables):
      spec = specs[k]
      spec = synth.TableSpec(f"table_{g}", spec.vocab, spec.dim, spec.dtype,
                             spec.combine, spec.weighted)
      rows, _, _ = synth.synth_table(xse._capi.DT_BF16, VOCAB, DIM, SEED, g)
      self.specs.append(spec)
      self.tables.append(rows)
      self.engine.add_table(spec.name, rows, spec.combine, adopt=True)
      self.engine.register_feature(spec.name, spec.name)
    self.inputs = []
    for v in range(ROTATE):
      batch = []
      for k, spec in enumerate(self.specs):
        batch.append(synth.synth_batch(spec, self.global_tables[k], BATCH,
                                       BAG, BAG, SEED, 0.0, variant=v))
      self.inputs.append(batch)
    self.status = xse.Status(NUM_TABLES * world)
    self.pooler = sharding.engine_pooler(self.engine, self.status)
    self.exchange = None
    if world == 1:
      self.pooled = [torch.empty((BATCH, NUM_TABLES, DIM), dtype=torch.float32,
                                 device="cuda") for _ in range(ROTATE)]
      self.requests = [self._requests(self.inputs[v], self.pooled[v])
                       for v in range(ROTATE)]
    else:
      # The C ABI's sharded execution over the engine's own NCCL
      # communicator (include/xse_shard.h).
      self.comm = sharding.ShardComm(torch.cuda.current_device(), self.plan)
      self.exchange = sharding.ShardedExchange(self.engine, self.comm,
                                               exchange, total, DIM, BATCH)
      self.steps = [self.exchange.prepare(self.features(v))
                    for v in range(ROTATE)]
      self.launches_per_step = exchange_launches(exchange, world)
    torch.cuda.synchronize()

  def features(self, v):
    return [(spec.name, fb.ids, fb.offsets, fb.weights)
            for spec, fb in zip(self.specs, self.inputs[v])]

  def _requests(self, batch, pooled):
    reqs = []
    for k, spec in enumerate(self.specs):
      fb = batch[k]
      reqs.append(self.xse.BagRequest(spec.name, fb.ids, fb.offsets,
                                      pooled[:, k, :], fb.weights,
                                      output_stride=NUM_TABLES * DIM))
    return self.xse.PreparedBatch(reqs)

  def step(self, i):
    v = i % ROTATE
    if self.world == 1:
      before = self.pooler.launches
      self.pooler(self.requests[v])
      return self.pooler.launches - before
    # Nothing reads the received rows here: each step's barrier overlaps
    # the next step's pooling; finish() waits for the last one.
    self.exchange.run(self.steps[v], defer=True)
    return self.launches_per_step

  def check(self):
    """Waits and raises the first error of the executions so far."""
    if self.world == 1:
      self.status.wait()
    else:
      self.exchange.check()

  def run_exchange(self, v):
    """One exchange whose output is ready on the current stream."""
    return self.exchange.run(self.steps[v])

  def finish(self):
    """Orders the current stream after every exchange issued so far."""
    if self.world > 1:
      self.exchange.ready()

  def ids_per_step(self):
    return NUM_TABLES * BATCH * BAG

  def parity_items(self, v):
    """The tables' pooled rows of variant v (N=1) for check_parity."""
    out = []
    for k, spec in enumerate(self.specs):
      fb = self.inputs[v][k]
      out.append({
          "dtype": self.xse._capi.DT_BF16, "stream": self.global_tables[k],
          "dim": DIM, "combine": spec.combine,
          "ids": fb.ids.cpu().numpy(), "offsets": fb.offsets.cpu().numpy(),
          "weights": None if fb.weights is None else fb.weights.cpu().numpy(),
          "window": None, "output": self.pooled[v][:, k, :]})
    return out

  def close(self):
    if self.world > 1:
      self.exchange.check()
      self.exchange.close()
      self.comm.close()
    self.status.close()
    self.engine.close()


def exchange_launches(mode, world, chunks=1):
  """Own kernels one sharded step launches: validation + pooling per group,
  plus the peer barrier (peer) or the reorder of received blocks (NCCL
  table-wise modes)."""
  if world == 1:
    return 2
  if mode == "peer":
    return 3
  if mode == "a2a":
    return 3
  if mode == "pipelined":
    return 2 * world + 1
  return 2 * chunks


def multi_table_config(world, exchange):
  return {
      "workload": WORKLOAD,
      "global_batch": BATCH,
      "tables_per_gpu": NUM_TABLES,
      "tables_total": NUM_TABLES * world,
      "accumulate": "fp32",
      "parallelism": ("single GPU" if world == 1 else
                      f"table-wise x{world} (table t on rank t mod "
                      f"{world}), pooled sample blocks returned to "
                      "their owners by " +
                      {"pipelined": "per-block NCCL send/recv "
                                    "overlapped with the pooling",
                       "a2a": "one NCCL all-to-all",
                       "peer": "the pooling kernel's own stores into "
                               "the owners' buffers over NVLink (CUDA "
                               "IPC) and a flag barrier"}[exchange]),
      "l2": "inputs larger than L2: 1.0 GB of tables per GPU and "
            f"{ROTATE} rotating id/offset/weight sets",
      "validation": "strict (separate validation kernel each step)",
  }


class OperatorHostInputs:
  """End-to-end measurement through the reference-facing operator: one
  CpuEmbeddingLookupTransform over the workload's features, called with
  host buffers in pinned memory (int64 ids, int32 row pointers, fp32
  weights) as a serving caller holds them. Each call copies the inputs to
  the device, validates, pools, and copies every pooled [batch, dim] fp32
  output back into pinned host buffers before it returns.

  tables: (name, rows, combine, scale, bias, vocab, row_begin, row_end) of
  the device tables (adopted by the operator's own resource); sets[v]: per
  table (ids, offsets, weights) device tensors of input variant v."""

  def __init__(self, xse, tables, sets, batch, dim):
    ops = xse.ops
    self.resource = ops.CpuEmbeddingResource.empty(torch.cuda.current_device())
    engine = self.resource.engine
    names = []
    for name, rows, combine, scale, bias, vocab, lo, hi in tables:
      engine.add_table(name, rows, combine, scale=scale, bias=bias,
                       vocab=vocab, row_begin=lo, row_end=hi, adopt=True)
      engine.register_feature(name, name)
      names.append(name)
    self.transform = ops.CpuEmbeddingLookupTransform(self.resource, names,
                                                     embedding_dim=dim)
    self.sets = []
    for feats in sets:
      ids_l, rp_l, w_l = [], [], []
      for ids_t, offs_t, w_t in feats:
        ids = ops.PinnedBuffer((ids_t.numel(),), np.int64)
        ids.array[:] = ids_t.cpu().numpy()
        rp = ops.PinnedBuffer((offs_t.numel(),), np.int32)
        rp.array[:] = offs_t.cpu().numpy()
        if w_t is not None:
          w = ops.PinnedBuffer((w_t.numel(),), np.float32)
          w.array[:] = w_t.cpu().numpy()
        else:
          w = ops.PinnedBuffer((0,), np.float32)
        ids_l.append(ids)
        rp_l.append(rp)
        w_l.append(w)
      self.sets.append((ids_l, rp_l, w_l))
    ids_l, rp_l, w_l = self.sets[0]
    self.h2d_bytes = sum(b.array.nbytes for b in ids_l + rp_l + w_l)
    self.d2h_bytes = batch * len(tables) * dim * 4
    self.prepared = [ops.PreparedInputs(*bufs) for bufs in self.sets]

  def step(self, i, stream=None):
    prepared = self.prepared[i % len(self.prepared)]
    outs = self.transform.output_array()
    self.transform.run_prepared(prepared, outs, stream=stream)
    self.transform.free_outputs(outs)

  def run(self, steps, threads):
    """`steps` synchronous transform calls spread over `threads` host
    threads, each on its own stream (concurrent requests, as a server issues
    them): one call's input copies overlap another's output copies. Returns
    the elapsed ms between events on the caller's stream that bracket every
    call (the join waits for each thread's stream)."""
    device = torch.cuda.current_device()
    main = torch.cuda.current_stream()
    streams = [torch.cuda.Stream() for _ in range(threads)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(main)
    for st in streams:
      st.wait_event(start)
    errors = []

    def worker(t):
      try:
        torch.cuda.set_device(device)
        for i in range(t, steps, threads):
          self.step(i, streams[t])
      except Exception as e:  # pylint: disable=broad-except
        errors.append(e)

    pool = [threading.Thread(target=worker, args=(t,)) for t in range(threads)]
    for th in pool:
      th.start()
    for th in pool:
      th.join()
    if errors:
      raise errors[0]
    for st in streams:
      main.wait_stream(st)
    end.record(main)
    torch.cuda.synchronize()
    return start.elapsed_time(end)

  def close(self):
    for bufs in self.sets:
      for lst in bufs:
        for b in lst:
          b.close()
    self.transform.close()
    self.resource.close()


class ShardedHostInputs:
  """End-to-end measurement through the sharded exchange (N > 1): each step
  copies this rank's inputs (ids, offsets, weights of the tables it pools,
  for the whole batch) from pinned host memory into the device tensors the
  exchange's request groups read, runs the exchange (pooling + the return
  of every sample block to its owner), and copies this rank's received
  pooled rows back into pinned host memory before the next step."""

  def __init__(self, run, device_sets, out_numel):
    self.run_exchange = run
    self.device_sets = device_sets
    self.host_sets = gather_inputs(device_sets)
    self.h2d_bytes = sum(tensor_bytes(f) for f in self.host_sets[0])
    self.out = torch.empty(out_numel, dtype=torch.float32).pin_memory()
    self.d2h_bytes = self.out.numel() * 4

  def step(self, i):
    v = i % len(self.device_sets)
    for dev_f, host_f in zip(self.device_sets[v], self.host_sets[v]):
      for d, h in zip(dev_f, host_f):
        if d is not None:
          d.copy_(h, non_blocking=True)
    out = self.run_exchange(v)
    self.out.copy_(out.reshape(-1), non_blocking=True)
    torch.cuda.current_stream().synchronize()


def timed_e2e(step, steps, world, local):
  """Max-over-ranks ms of `steps` synchronous end-to-end steps."""
  for i in range(3):
    step(i)
  ms, _ = timed_steps(lambda i: step(i), 0, steps, world, local)
  return ms


def cpu_baseline(wl, seconds):
  """Times the oracle (CPU restatement of the reference's threaded
  ExecuteEmbeddingBagBatch) on this host's cores over full batches of the
  same workload (same tables and ids, copied to host)."""
  oracle = load_oracle()
  cores = oracle.host_cores()
  bags = []
  for k, spec in enumerate(wl.specs):
    bits = wl.tables[k].view(torch.int16).cpu().numpy().view(np.uint16)
    fb = wl.inputs[0][k]
    bags.append(oracle.Bag(
        bits, fb.ids.cpu().numpy(), fb.offsets.cpu().numpy(),
        None if fb.weights is None else fb.weights.cpu().numpy(),
        spec.combine, oracle.BF16))
  oracle.embedding_bag_batch(bags, num_threads=cores)  # warm-up
  reps, t0 = 0, time.perf_counter()
  while True:
    oracle.embedding_bag_batch(bags, num_threads=cores)
    reps += 1
    el = time.perf_counter() - t0
    if el >= seconds:
      break
  ids = reps * wl.ids_per_step()
  return {"value": ids / el, "unit": "ids/s", "cores": cores, "kind": "port",
          "sample": f"{reps} full batches (8 tables x 8192 bags x 20 ids, "
                    f"bf16 rows widened to fp32) in {el:.1f} s"}


# ---------------------------------------------------------------------------
# The other reference configurations.

CONFIGS = {
    "zipf_single": dict(
        desc="zipf_single: 1 fp32 table 1,000,000 x 64, batch 4096, bag "
             "lengths U[1,32], Zipf(1.05) ids, sum pooling",
        tables=1, dtype="f32", vocab=1_000_000, dim=64, batch=4096,
        lengths=(1, 32), alpha=1.05, sharding="replica", rotate=64,
        check_bags=4096, cpu_seconds=3.0),
    "sharded_tablewise": dict(
        desc="sharded_tablewise: 64 bf16 tables 20,000,000 x 128 (327 GB) "
             "placed table-wise, 8 tables per GPU (table t on rank t mod N; "
             "the 8-table per-GPU slice at N=1), batch 65536, bag lengths "
             "U[1,64], Zipf(1.1) ids, sum pooling",
        tables_per_gpu=8, dtype="bf16", vocab=20_000_000, dim=128,
        batch=65536, lengths=(1, 64), alpha=1.1, sharding="table", rotate=2,
        check_bags=1024, cpu_seconds=3.0),
    "int8_rowwise": dict(
        desc="int8_rowwise: 26 int8 row-wise tables 10,000,000 x 256 with "
             "per-row fp32 scale U(1e-3,1e-2) and bias U(-0.1,0.1), rows "
             "split row-wise over the N ranks, batch 32768, bag lengths "
             "U[1,80], Zipf(1.05) ids, sum pooling with in-kernel dequant, "
             "partial sums reduce-scattered",
        tables=26, dtype="i8", vocab=10_000_000, dim=256, batch=32768,
        lengths=(1, 80), alpha=1.05, sharding="row", rotate=2,
        check_bags=256, cpu_seconds=3.0),
}
_ELEM = {"f32": 4, "bf16": 2, "i8": 1}
CONFIG_TABLE_STREAM = 200  # synth stream of global table g: 200 + g


class ConfigWorkload:
  """Tables, inputs and the exchange of one CONFIGS entry on this rank.

  sharding "replica": every rank pools its own copy (weak scaling, no
  exchange); "table": tables_per_gpu tables per rank, table-wise exchange
  of the pooled sample blocks; "row": every table's rows split over the
  ranks, partial sums reduce-scattered."""

  def __init__(self, xse, cfg, rank, world, exchange, max_rows=None):
    from xla_serving_b200 import sharding, synth  # pylint: disable=import-outside-toplevel
    C = xse._capi
    if max_rows:  # smaller tables, for profiler captures
      cfg = dict(cfg, vocab=min(cfg["vocab"], int(max_rows)))
    self.xse, self.cfg, self.world, self.rank = xse, cfg, world, rank
    self.sharding = sharding
    dt = {"f32": C.DT_F32, "bf16": C.DT_BF16, "i8": C.DT_I8_ROWWISE}[
        cfg["dtype"]]
    self.dtype = dt
    self.engine = xse.EmbeddingEngine(torch.cuda.current_device())
    mode = cfg["sharding"]
    # A replica rank pools its tables alone: a plan of one.
    self.plan = (sharding.ShardPlan(1, 0) if mode == "replica" else
                 sharding.ShardPlan(world, rank))
    if mode == "table":
      num_tables = cfg["tables_per_gpu"] * world
    else:
      num_tables = cfg["tables"]
    self.num_tables = num_tables
    rowwise = mode == "row"
    local = (list(range(num_tables)) if rowwise or mode == "replica" else
             self.plan.tables_of(rank, num_tables))
    self.local = local
    vocab, dim = cfg["vocab"], cfg["dim"]
    lo, hi = self.plan.row_window(vocab) if rowwise else (0, vocab)
    self.window = (lo, hi)
    self.tables = []
    for g in local:
      rows, scale, bias = synth.synth_table(dt, vocab, dim, SEED,
                                            CONFIG_TABLE_STREAM + g,
                                            row0=lo, nrows=hi - lo)
      name = f"t{g}"
      self.engine.add_table(name, rows, "SUM", scale=scale, bias=bias,
                            vocab=vocab, row_begin=lo if rowwise else 0,
                            row_end=hi if rowwise else 0, adopt=True)
      self.tables.append((name, rows, "SUM", scale, bias, vocab,
                          lo if rowwise else 0, hi if rowwise else 0))
      self.engine.register_feature(name, name)
    self.inputs = []
    self.nnz = []
    for v in range(cfg["rotate"]):
      feats = []
      nnz = 0
      for g in local:
        spec = synth.TableSpec(f"t{g}", vocab, dim, dt, "SUM")
        # Replica ranks draw their own batches.
        stream = CONFIG_TABLE_STREAM + g + (
            100_000 * rank if mode == "replica" else 0)
        fb = synth.synth_batch(spec, stream, cfg["batch"], cfg["lengths"][0],
                               cfg["lengths"][1], SEED, cfg["alpha"],
                               variant=v)
        feats.append((spec.name, fb.ids, fb.offsets, None))
        nnz += fb.ids.numel()
      self.inputs.append(feats)
      self.nnz.append(nnz)
    # The C ABI's sharded execution (include/xse_shard.h) over the engine's
    # own NCCL communicator; a replica rank is a job of one rank.
    w = self.plan.world
    self.chunks = 2 if rowwise and w > 1 else 1
    self.mode_name = "row" if rowwise else exchange
    self.comm = sharding.ShardComm(torch.cuda.current_device(), self.plan)
    self.exchange = sharding.ShardedExchange(
        self.engine, self.comm, self.mode_name,
        num_tables if mode == "table" else len(local), dim, cfg["batch"],
        chunks=self.chunks)
    self.steps = [self.exchange.prepare(f) for f in self.inputs]
    self.launches_per_step = exchange_launches(self.mode_name, w,
                                               self.chunks)
    # Pooling launches per step (row-wise chunks and pipelined destination
    # blocks: one group each).
    self.pool_groups = (self.chunks if rowwise else
                        w if self.mode_name == "pipelined" and w > 1 else 1)
    # Table-wise at N > 1: the same batch arriving data-parallel (every
    # table's ids for this rank's samples) for the separately timed ids
    # all-to-all that would feed the owners.
    self.ids_a2a, self.dp_input = None, None
    if mode == "table" and world > 1:
      block = self.plan.block_size(cfg["batch"])
      self.dp_input = []
      for g in range(num_tables):
        spec = synth.TableSpec(f"t{g}", vocab, dim, dt, "SUM")
        fb = synth.synth_batch(spec, 5000 + 97 * rank + g, block,
                               cfg["lengths"][0], cfg["lengths"][1], SEED,
                               cfg["alpha"])
        self.dp_input.append((spec.name, fb.ids, fb.offsets, None))
      self.ids_a2a = sharding.IdsAllToAll(self.plan, cfg["batch"],
                                          num_tables, device="cuda")
    torch.cuda.synchronize()

  def run(self, v, wait=True):
    """One step of input variant v; returns this rank's pooled rows."""
    return self.exchange.run(self.steps[v], defer=not wait)

  def step(self, i):
    self.run(i % len(self.steps), wait=False)
    return self.launches_per_step

  def finish(self):
    self.exchange.ready()

  def outputs(self):
    """[batch, local tables, dim] pooled rows of the last step (one rank's
    whole batch: N=1, or a replica)."""
    return self.exchange.recv

  def parity_items(self, v):
    out = self.outputs()
    rowwise = self.cfg["sharding"] == "row"
    items = []
    for k, g in enumerate(self.local):
      _, ids, offsets, _ = self.inputs[v][k]
      items.append({
          "dtype": self.dtype, "stream": CONFIG_TABLE_STREAM + g,
          "dim": self.cfg["dim"], "combine": "SUM",
          "ids": ids.cpu().numpy(), "offsets": offsets.cpu().numpy(),
          "weights": None, "window": self.window if rowwise else None,
          "output": out[:, k, :]})
    return items

  def ids_per_step(self, v):
    """Ids pooled by the whole job in one step: every rank's table-wise ids
    (or replica batches); row-wise ranks all see the same ids."""
    return self.nnz[v]

  def pool_bytes(self, v):
    """Algorithmic bytes of variant v's pooling on this rank: every id's row
    (int8 rows plus their 8-byte scale/bias) and id, the offsets, the fp32
    outputs."""
    cfg = self.cfg
    row = cfg["dim"] * _ELEM[cfg["dtype"]] + (8 if cfg["dtype"] == "i8" else 0)
    t = len(self.local)
    return (self.nnz[v] * (row + 8) + (cfg["batch"] + 1) * 8 * t +
            cfg["batch"] * t * cfg["dim"] * 4)

  def close(self):
    self.exchange.check()
    self.exchange.close()
    self.comm.close()
    self.engine.close()


def config_cpu_baseline(wl, seconds):
  """The oracle on this host's cores over a bounded sample: the first
  table's first 4M rows (or all rows) copied to the host, Zipf ids over that
  subset, the config's bag lengths, for about `seconds`."""
  oracle = load_oracle()
  from xla_serving_b200 import synth  # pylint: disable=import-outside-toplevel
  cfg = wl.cfg
  cores = oracle.host_cores()
  sub = min(cfg["vocab"], 4_000_000)
  rows, scale, bias = synth.synth_table(wl.dtype, cfg["vocab"], cfg["dim"],
                                        SEED, CONFIG_TABLE_STREAM, nrows=sub)
  if cfg["dtype"] == "bf16":
    table = rows.view(torch.int16).cpu().numpy().view(np.uint16)
    odt = oracle.BF16
  elif cfg["dtype"] == "i8":
    table = rows.cpu().numpy()
    odt = oracle.I8_ROWWISE
  else:
    table = rows.cpu().numpy()
    odt = oracle.F32
  sc = None if scale is None else scale.cpu().numpy()
  bi = None if bias is None else bias.cpu().numpy()
  del rows
  spec = synth.TableSpec("cpu", sub, cfg["dim"], wl.dtype, "SUM")
  bags = []
  for k in range(4):
    fb = synth.synth_batch(spec, 900 + k, cfg["batch"], cfg["lengths"][0],
                           cfg["lengths"][1], SEED, cfg["alpha"])
    bags.append(oracle.Bag(table, fb.ids.cpu().numpy(),
                           fb.offsets.cpu().numpy(), None, "SUM", odt, sc, bi))
  oracle.embedding_bag_batch(bags[:1], num_threads=cores)
  reps, t0 = 0, time.perf_counter()
  while True:
    oracle.embedding_bag_batch([bags[reps % 4]], num_threads=cores)
    reps += 1
    el = time.perf_counter() - t0
    if el >= seconds:
      break
  ids = sum(len(bags[i % 4].ids) for i in range(reps))
  return {"value": ids / el, "unit": "ids/s", "cores": cores, "kind": "port",
          "sample": f"{reps} batches of {cfg['batch']} bags over the first "
                    f"{sub:,} rows of one table ({cfg['dtype']}"
                    f"{', dequantized per row' if cfg['dtype'] == 'i8' else ''}"
                    f") in {el:.1f} s"}


def measure_config(xse, args, name, world, rank, local, max_rows=None):
  """One CONFIGS workload at N GPUs: device rate, kernel roofline,
  end-to-end rate with host buffers, and (N=1) CPU baseline and parity."""
  cfg = CONFIGS[name]
  wl = ConfigWorkload(xse, cfg, rank, world, args.exchange, max_rows)
  mode = cfg["sharding"]
  for i in range(args.warmup):
    wl.step(i)
  wl.finish()
  wl.exchange.check()
  ms, launches = timed_steps(wl.step, args.warmup, args.steps, world, local,
                             wl.finish)
  wl.exchange.check()
  pool_ms, pool_n, val_ms = kernel_timing(
      wl.engine, wl.step, args.warmup + args.steps,
      max(KERNEL_TIMING_LAUNCHES // wl.pool_groups, 8), wl.finish)
  wl.exchange.check()
  rot = len(wl.nnz)
  ids_rank = sum(wl.nnz[(args.warmup + i) % rot] for i in range(args.steps))
  ids = ids_rank if mode == "row" else sum_over_ranks(ids_rank, world)
  pool_bytes = sum(wl.pool_bytes(i % rot) for i in range(rot)) / rot
  pool_step_ms = pool_ms * wl.pool_groups
  peak, peak_kind = measured_peaks()
  achieved = pool_bytes / (pool_step_ms / 1000.0) / 1e9

  # End to end with host buffers.
  if world == 1 or mode == "replica":
    host = OperatorHostInputs(
        xse, wl.tables,
        [[(f[1], f[2], f[3]) for f in feats] for feats in wl.inputs],
        cfg["batch"], cfg["dim"])
    warm = 4 * E2E_THREADS
    per_call = host.run(warm, E2E_THREADS) / warm
    per_call = max_over_ranks(per_call, world)
    e_steps = int(min(2000, max(16, E2E_TARGET_MS / max(per_call, 1e-3))))
    barrier(world, local)
    e_ms = max_over_ranks(host.run(e_steps, E2E_THREADS), world)
    e_path = ("CpuEmbeddingLookupTransform (xse_lookup_transform_run, C "
              f"ABI) over {len(wl.local)} features with pinned host "
              "inputs; H2D, validation, pooling and D2H of the outputs "
              f"inside each synchronous call; {E2E_THREADS} host threads")
    h2d, d2h = host.h2d_bytes, host.d2h_bytes
    host.close()
  else:
    sh = ShardedHostInputs(
        lambda v: wl.run(v, wait=True),
        [[(f[1], f[2], f[3]) for f in feats] for feats in wl.inputs],
        wl.exchange.block * wl.exchange.num_tables * cfg["dim"])
    e_steps = max(4, args.steps // 2)
    e_ms = timed_e2e(sh.step, e_steps, world, local)
    e_path = ("sharded exchange with host buffers: this rank's ids and "
              "offsets copied from pinned memory, pooling plus the " +
              ("reduce-scatter" if mode == "row" else
               f"{args.exchange} exchange") +
              ", this rank's pooled rows copied back, synchronous per step")
    h2d, d2h = sh.h2d_bytes, sh.d2h_bytes
  e_ids_rank = sum(wl.nnz[i % rot] for i in range(e_steps))
  e_ids = e_ids_rank if mode == "row" else sum_over_ranks(e_ids_rank, world)

  base = parity = None
  if world == 1 and not args.no_cpu_baseline:
    base = config_cpu_baseline(wl, cfg["cpu_seconds"])
    v = 0
    wl.run(v)
    wl.exchange.check()
    parity = check_parity(wl.parity_items(v), cfg["check_bags"])
  ids_a2a = None
  if wl.ids_a2a is not None:
    # Timed on its own: extents, their all-to-all and host read, the pack
    # launch and the all-to-alls of offsets and ids, every step.
    for _ in range(3):
      wl.ids_a2a.run(wl.dp_input)
    a2a_steps = 10
    a2a_ms, _ = timed_steps(lambda i: wl.ids_a2a.run(wl.dp_input), 0,
                            a2a_steps, world, local)
    ids_a2a = {"ms_per_step": a2a_ms / a2a_steps, "steps": a2a_steps,
               "ids_per_rank": sum(int(f[1].numel()) for f in wl.dp_input),
               "bytes_sent_per_rank": wl.ids_a2a.bytes_last,
               "note": "data-parallel input (every table's ids for this "
                       "rank's samples) moved to the table owners; timed "
                       "apart from the pooling"}
  result = {
      "metric": "embedding-bag ids/sec", "value": ids / (ms / 1000.0),
      "unit": "ids/s", "n_gpus": world, "steps": args.steps,
      "warmup": args.warmup, "ms_per_step": ms / args.steps,
      "higher_is_better": True,
      "scaling": "weak" if mode in ("replica", "table") else "strong",
      "dtype": cfg["dtype"], "data": "synthetic (seeded counter RNG)",
      "config": {"workload": cfg["desc"] + (
                     f" (rows capped at {int(max_rows):,} for a profiler "
                     "capture)" if max_rows else ""),
                 "global_batch": cfg["batch"] * (
                     world if mode == "replica" else 1),
                 "tables_total": wl.num_tables,
                 "tables_per_gpu": len(wl.local),
                 "rows_per_gpu": wl.window[1] - wl.window[0],
                 "parallelism": ("single GPU" if world == 1 else
                                 {"replica": f"{world} independent replicas",
                                  "row": "row-wise windows + NCCL "
                                         "reduce-scatter",
                                  "table": f"table-wise, {args.exchange} "
                                           "exchange"}[mode]),
                 "l2": f"{cfg['rotate']} rotating input sets; tables "
                       "far larger than L2 (Zipf hot rows hit it)"},
      "roofline": {
          "bound": "hbm", "achieved": achieved, "peak": peak,
          "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
          "traffic": None,
          "algorithmic_bytes_per_step": pool_bytes,
          "pool_ms_per_step": pool_step_ms, "avg_launch_ms": pool_ms,
          "timed_launches": pool_n,
          "note": "Zipf hot rows hit L2: algorithmic bytes count every id's "
                  "row with no cache credit"},
      "e2e": {"value": e_ids / (e_ms / 1000.0), "unit": "ids/s",
              "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
              "path": e_path},
      "gpu_launches": launches,
      "validation": validation_share(val_ms, ms / args.steps),
      "cpu_baseline": base,
      "parity": parity,
  }
  if ids_a2a is not None:
    result["ids_all_to_all"] = ids_a2a
  wl.close()
  del wl
  torch.cuda.synchronize()
  torch.cuda.empty_cache()
  return result


# ---------------------------------------------------------------------------
# DLRM forward.

# DLRM forward workload: 26 fp32 tables x 128, rows log-uniform in
# [1e4, 1e7], batch 16384, bag lengths U[1,100], Zipf(1.05) ids, sum pooling,
# 13 dense features N(0,1), bottom MLP 13-512-256-128, dot interaction (479),
# top MLP 479-1024-1024-512-256-1 with sigmoid. Ids and row pointers are
# int32, as the reference's DLRM bundle feeds them.
DLRM_TABLES = 26
DLRM_DIM = 128
DLRM_BATCH = 16384
DLRM_LEN = (1, 100)
DLRM_ALPHA = 1.05
DLRM_ROTATE = 4
DLRM_TABLE_STREAM = 100  # synth table-stream offset (independent of above)
DLRM_CHECK_SAMPLES = 1024
DLRM_WORKLOAD = ("dlrm_forward: 26 fp32 tables x 128 (rows log-uniform in "
                 "[1e4, 1e7]), batch 16384, bag lengths U[1,100], Zipf(1.05) "
                 "int32 ids and row pointers, sum pooling; 13 dense features "
                 "N(0,1); bottom MLP 13-512-256-128 ReLU; dot interaction "
                 "128+351=479; top MLP 479-1024-1024-512-256-1 sigmoid; fp32")


class DlrmWorkload:
  """One DLRM forward per step on this rank's GPU (a full replica: every
  rank holds all 26 tables and runs its own batch)."""

  def __init__(self, xse, rank, max_rows=None):
    from xla_serving_b200 import dlrm, synth  # pylint: disable=import-outside-toplevel
    self.xse = xse
    self.engine = xse.EmbeddingEngine(torch.cuda.current_device())
    self.rows = synth.log_uniform_rows(DLRM_TABLES, 1e4, 1e7, SEED)
    if max_rows:  # smaller tables, for profiler captures
      self.rows = [min(r, int(max_rows)) for r in self.rows]
    names, self.tables = [], []
    for t in range(DLRM_TABLES):
      rows, _, _ = synth.synth_table(xse._capi.DT_F32, self.rows[t], DLRM_DIM,
                                     SEED, DLRM_TABLE_STREAM + t)
      name = f"sparse_{t}"
      self.tables.append(rows)
      self.engine.add_table(name, rows, "SUM", adopt=True)
      self.engine.register_feature(name, name)
      names.append(name)
    # Dense layers as three TF32 tensor-core GEMMs over hi/lo split operands
    # (fp32-level accuracy; the DLRM tests hold them to the fp32 layer's
    # tolerance).
    self.model = dlrm.DLRM(self.engine, names, dim=DLRM_DIM, seed=SEED,
                           math=dlrm.MATH_TF32X3)
    gen = torch.Generator(device="cuda").manual_seed(SEED + rank)
    self.sets = []
    self.nnz = []
    self.streams = []
    for v in range(DLRM_ROTATE):
      ids, offsets = [], []
      for t in range(DLRM_TABLES):
        spec = synth.TableSpec(names[t], self.rows[t], DLRM_DIM,
                               xse._capi.DT_F32, "SUM")
        fb = synth.synth_batch(spec, DLRM_TABLE_STREAM + 64 * rank + t,
                               DLRM_BATCH, DLRM_LEN[0], DLRM_LEN[1], SEED,
                               DLRM_ALPHA, variant=v)
        ids.append(fb.ids.to(torch.int32))
        offsets.append(fb.offsets.to(torch.int32))
      reqs, _ = self.model.requests(ids, offsets)
      dense = torch.randn((DLRM_BATCH, 13), generator=gen, device="cuda")
      self.sets.append((dense, reqs, ids, offsets))
      self.nnz.append(sum(int(i.numel()) for i in ids))
    self.status = xse.Status(DLRM_TABLES)
    torch.cuda.synchronize()

  def step(self, i):
    dense, reqs, _, _ = self.sets[i % DLRM_ROTATE]
    self.model.forward(dense, requests=reqs, status=self.status)
    # Own kernels: the fused pooling + interaction launch (fused checks; or
    # pooling and the interaction kernel), the sigmoid head and one operand
    # split per split-TF32 layer whose input the interaction does not split
    # (the GEMMs are cuBLASLt's).
    fused = self.model.fused_interaction
    return (1 if fused else 2) + 1 + self.model.tower.split_launches(fused)

  def pool_bytes(self, v):
    """Algorithmic bytes of variant v's timed kernel: every id's row and id
    (int32), the int32 offsets, and either the pooled [B, 26, 128] fp32
    output or -- fused with the interaction -- the bottom-MLP rows read and
    the [B, 480] interaction rows written (twice: TF32 hi and lo parts)."""
    lookup = (self.nnz[v] * (DLRM_DIM * 4 + 4) +
              (DLRM_BATCH + 1) * 4 * DLRM_TABLES)
    if self.model.fused_interaction:
      return lookup + DLRM_BATCH * (
          DLRM_DIM + self.model.tower.interaction_bytes_per_row() // 4) * 4
    return lookup + DLRM_BATCH * DLRM_TABLES * DLRM_DIM * 4

  def parity(self, v, count):
    """Sampled samples of variant v against the oracle: their pooled rows
    (through the unfused pooling of the same requests), the interaction rows
    the fused kernel wrote, and the predictions (float64 tower)."""
    oracle = load_oracle()
    dense, reqs, ids, offsets = self.sets[v]
    pred = self.model.forward(dense, requests=reqs).clone()
    tower = self.model.tower
    x = tower.bottom_output(DLRM_BATCH).clone()
    # The interaction rows (the forward writes them as split operands,
    # which later layers' splits overwrite): once as values, once split.
    inter = torch.empty((DLRM_BATCH, tower.width_stride), device="cuda")
    self.engine.execute_interaction(reqs, x, inter, fused=True)
    hi, lo = torch.empty_like(inter), torch.empty_like(inter)
    self.engine.execute_interaction(reqs, x, hi, fused=True, out_lo=lo)
    split_exact = bool(torch.equal(hi + lo, inter))
    torch.cuda.synchronize()
    pooled = self.model.pooled_buffer(DLRM_BATCH)
    self.engine.execute_batch(reqs)
    items = []
    for t in range(DLRM_TABLES):
      items.append({"dtype": self.xse._capi.DT_F32,
                    "stream": DLRM_TABLE_STREAM + t, "dim": DLRM_DIM,
                    "combine": "SUM", "ids": ids[t].cpu().numpy(),
                    "offsets": offsets[t].cpu().numpy(), "weights": None,
                    "window": None, "output": pooled[:, t, :]})
    # One sample set for every table, so the interaction can be checked.
    samples = oracle.sampled_bags(DLRM_BATCH, count, SEED + 17)
    t0 = time.perf_counter()
    cores = oracle.host_cores()
    want_pooled = np.zeros((len(samples), DLRM_TABLES, DLRM_DIM), np.float32)
    pooled_summary = {"ok": True, "bit_exact": True, "max_abs_err": 0.0,
                      "mismatched": 0}
    idx = torch.from_numpy(samples).cuda()
    for t, it in enumerate(items):
      want, _ = oracle.pool_sampled(
          it["dtype"], SEED, it["stream"], DLRM_DIM, "SUM", it["ids"],
          it["offsets"], None, samples, num_threads=cores)
      want_pooled[:, t, :] = want
      r = oracle.compare_pooled(it["output"][idx].cpu().numpy(), want)
      pooled_summary["ok"] &= r["ok"]
      pooled_summary["bit_exact"] &= r["bit_exact"]
      pooled_summary["mismatched"] += r["mismatched"]
      pooled_summary["max_abs_err"] = max(pooled_summary["max_abs_err"],
                                          r["max_abs_err"])
    xs = x[idx].cpu().numpy()
    want_inter = oracle.dot_interaction(xs, want_pooled)
    bound = oracle.dot_interaction(np.abs(xs), np.abs(want_pooled))
    width = want_inter.shape[1]
    got_inter = inter[idx][:, :width].cpu().numpy()
    err = np.abs(got_inter.astype(np.float64) - want_inter)
    inter_ok = bool((err <= 1e-4 * bound + 1e-30).all())
    dense_s = dense[idx].cpu().numpy()
    want_pred = self.model.tower.reference_forward(dense_s, want_pooled)
    pred_err = float(np.abs(pred[idx].cpu().numpy() - want_pred).max())
    return {
        "samples_checked": int(len(samples)), "tables": DLRM_TABLES,
        "pooled": pooled_summary,
        "interaction": {"ok": inter_ok, "max_abs_err": float(err.max()),
                        "rule": "|err| <= 1e-4 x sum|z_i z_j|",
                        "split_operands_exact": split_exact},
        "predictions": {"ok": pred_err <= 1e-4, "max_abs_err": pred_err,
                        "rule": "|err| <= 1e-4 (float64 tower on the "
                                "oracle's pooled rows)"},
        "ok": (pooled_summary["ok"] and inter_ok and split_exact and
               pred_err <= 1e-4),
        "seconds": time.perf_counter() - t0,
    }

  def close(self):
    self.status.close()
    self.engine.close()


class DlrmHostInputs:
  """End-to-end DLRM forward through DLRM.forward with host inputs: per step
  the int32 ids and row pointers and the dense features are copied from
  pinned host memory into the device tensors the requests point at, and the
  predictions are read back into pinned host memory."""

  def __init__(self, wl):
    self.wl = wl
    self.host = []
    for dense, _, ids, offsets in wl.sets:
      self.host.append(([x.cpu().pin_memory() for x in ids],
                        [x.cpu().pin_memory() for x in offsets],
                        dense.cpu().pin_memory()))
    self.h2d_bytes = sum(x.numel() * x.element_size()
                         for lst in self.host[0][:2] for x in lst)
    self.h2d_bytes += self.host[0][2].numel() * 4
    self.pred = torch.empty(DLRM_BATCH, dtype=torch.float32).pin_memory()
    self.d2h_bytes = DLRM_BATCH * 4

  def step(self, i):
    v = i % DLRM_ROTATE
    dense, reqs, ids, offsets = self.wl.sets[v]
    h_ids, h_offs, h_dense = self.host[v]
    for dst, src in zip(ids, h_ids):
      dst.copy_(src, non_blocking=True)
    for dst, src in zip(offsets, h_offs):
      dst.copy_(src, non_blocking=True)
    dense.copy_(h_dense, non_blocking=True)
    pred = self.wl.model.forward(dense, requests=reqs)
    self.pred.copy_(pred, non_blocking=True)
    torch.cuda.current_stream().synchronize()


def measure_dlrm(xse, args, world, local, check=True):
  """Samples/s of the DLRM forward (whole job: every rank runs its own
  batch), its pooled-lookup roofline, its end-to-end rate and (N=1) a
  sampled parity check."""
  wl = DlrmWorkload(xse, int(os.environ.get("RANK", "0")), args.dlrm_max_rows)
  host = DlrmHostInputs(wl)
  for i in range(args.warmup):
    wl.step(i)
  wl.status.wait()
  ms, launches = timed_steps(wl.step, args.warmup, args.dlrm_steps, world,
                             local)
  wl.status.wait()
  pool_avg, pool_n, _ = kernel_timing(wl.engine, wl.step,
                                   args.warmup + args.dlrm_steps,
                                   KERNEL_TIMING_LAUNCHES)
  wl.status.wait()
  samples = sum_over_ranks(DLRM_BATCH * args.dlrm_steps, world)
  ids = sum_over_ranks(sum(wl.nnz[(args.warmup + i) % DLRM_ROTATE]
                           for i in range(args.dlrm_steps)), world)
  pool_bytes = sum(wl.pool_bytes(v) for v in range(DLRM_ROTATE)) / DLRM_ROTATE
  peak, peak_kind = measured_peaks()
  e_steps = max(args.dlrm_steps // 4, 5)
  e_ms = timed_e2e(host.step, e_steps, world, local)
  e_samples = sum_over_ranks(DLRM_BATCH * e_steps, world)
  parity = None
  if check and world == 1 and not args.no_cpu_baseline:
    parity = wl.parity(0, DLRM_CHECK_SAMPLES)
  result = {
      "metric": "DLRM-fwd samples/sec",
      "value": samples / (ms / 1000.0),
      "unit": "samples/s",
      "n_gpus": world,
      "steps": args.dlrm_steps,
      "ms_per_step": ms / args.dlrm_steps,
      "ids_per_s": ids / (ms / 1000.0),
      "dtype": "fp32 (tables, pooling); interaction Gram and dense layers "
               "as 3xTF32 tensor-core MMAs (hi/lo split operands, "
               "fp32-level accuracy)",
      "parallelism": ("single GPU" if world == 1 else
                      f"{world} data-parallel replicas (tables replicated, "
                      "no collective)"),
      "config": {"workload": DLRM_WORKLOAD, "batch_per_gpu": DLRM_BATCH,
                 "table_rows": wl.rows,
                 "l2": f"{sum(wl.rows) * DLRM_DIM * 4 / 1e9:.1f} GB of tables "
                       f"and {DLRM_ROTATE} rotating input sets per GPU"},
      "pool_roofline": {
          "kernel": ("PoolInteractKernel<fp32> (pooled lookup + dot "
                     "interaction, split-TF32 mma.sync Gram)"
                     if wl.model.fused_interaction else
                     "PoolVecKernel<fp32, G=32, V=1, exact>"),
          "bound": "hbm", "achieved": pool_bytes / (pool_avg / 1000.0) / 1e9,
          "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
          "frac": pool_bytes / (pool_avg / 1000.0) / 1e9 / peak,
          "algorithmic_bytes_per_launch": pool_bytes,
          "avg_launch_ms": pool_avg, "timed_launches": pool_n,
          "note": "Zipf(1.05) hot rows hit L2, so algorithmic GB/s can "
                  "exceed DRAM bandwidth"},
      "gpu_launches": launches,
      "e2e": {"value": e_samples / (e_ms / 1000.0), "unit": "samples/s",
              "h2d_bytes_per_step": host.h2d_bytes,
              "d2h_bytes_per_step": host.d2h_bytes,
              "path": "DLRM.forward with int32 ids and row pointers and the "
                      "dense features copied from pinned host memory and "
                      "predictions copied back, synchronous per step"},
      "parity": parity,
  }
  wl.close()
  del wl, host
  torch.cuda.synchronize()
  torch.cuda.empty_cache()
  return result


# ---------------------------------------------------------------------------
# The reference's own DLRM bundle lookup (examples/dlrm/model_jce.py:28-84,
# export_jce.py:100-118,178-194): 26 fp32 tables of VOCAB_SIZES x 128,
# valency VALENCY[i] ids per example (214 in all), uniform ids, int32
# [B, valency] inputs, dense_lookup row pointers b * valency, SUM pooling.
REF_VOCAB = [400000, 39060, 17295, 7424, 20265, 3, 7122, 1543, 63, 400000,
             3067956, 405282, 10, 2209, 11938, 155, 4, 976, 14, 400000,
             400000, 400000, 590152, 12973, 108, 36]
REF_VALENCY = [3, 2, 1, 2, 6, 1, 1, 1, 1, 7, 3, 8, 1, 6, 9, 5, 1, 1, 1, 12,
               100, 27, 10, 3, 1, 1]
REF_DIM = 128
REF_BATCH = 16384   # device-side batch of the lookup
REF_BATCH_REQ = 128  # per-call batch of the reference's published figure
REF_TABLE_STREAM = 300
REF_ROTATE = 4
# XSE's C++ embedding kernel: 24,500 examples per core-second at B_req = 128
# (docs/benchmarks/dlrm_serving.md:240-244), on the reference's own host.
REF_PUBLISHED = 24500.0


class DlrmLookupWorkload:
  """The reference bundle's lookup on this GPU: tables, int32 dense ids."""

  def __init__(self, xse, rank):
    from xla_serving_b200 import synth  # pylint: disable=import-outside-toplevel
    C = xse._capi
    self.xse = xse
    self.engine = xse.EmbeddingEngine(torch.cuda.current_device())
    self.tables = []
    self.names = []
    for t, vocab in enumerate(REF_VOCAB):
      rows, _, _ = synth.synth_table(C.DT_F32, vocab, REF_DIM, SEED,
                                     REF_TABLE_STREAM + t)
      name = str(t)
      self.engine.add_table(name, rows, "SUM", adopt=True)
      self.engine.register_feature(name, name)
      self.tables.append((name, rows, "SUM", None, None, vocab, 0, 0))
      self.names.append(name)
    self.pooled = torch.empty((REF_BATCH, len(REF_VOCAB), REF_DIM),
                              dtype=torch.float32, device="cuda")
    self.sets = []
    for v in range(REF_ROTATE):
      feats = []
      for t, (vocab, val) in enumerate(zip(REF_VOCAB, REF_VALENCY)):
        ids = synth.synth_ids(REF_BATCH * val, vocab, SEED,
                              REF_TABLE_STREAM + 64 * rank + t + 1000 * v)
        rp = torch.arange(0, REF_BATCH * val + 1, val, dtype=torch.int32,
                          device="cuda")
        feats.append((ids.to(torch.int32), rp))
      self.sets.append(feats)
    self.requests = []
    for feats in self.sets:
      reqs = [xse.BagRequest(self.names[t], ids, rp, self.pooled[:, t, :],
                             None, output_stride=len(REF_VOCAB) * REF_DIM)
              for t, (ids, rp) in enumerate(feats)]
      self.requests.append(xse.PreparedBatch(reqs))
    self.status = xse.Status(len(REF_VOCAB))
    torch.cuda.synchronize()

  def step(self, i):
    self.engine.execute_batch(self.requests[i % REF_ROTATE],
                              status=self.status)
    return self.xse.last_launch_count()

  def bytes_per_step(self):
    nnz = REF_BATCH * sum(REF_VALENCY)
    return (nnz * (REF_DIM * 4 + 4) + (REF_BATCH + 1) * 4 * len(REF_VOCAB) +
            REF_BATCH * len(REF_VOCAB) * REF_DIM * 4)

  def parity_items(self, v):
    out = []
    for t, (ids, rp) in enumerate(self.sets[v]):
      out.append({"dtype": self.xse._capi.DT_F32,
                  "stream": REF_TABLE_STREAM + t, "dim": REF_DIM,
                  "combine": "SUM", "ids": ids.cpu().numpy(),
                  "offsets": rp.cpu().numpy(), "weights": None,
                  "window": None, "output": self.pooled[:, t, :]})
    return out

  def close(self):
    self.status.close()
    self.engine.close()


class DenseLookupHostInputs:
  """The bundle's serving call: CpuEmbeddingLookupTransform with
  dense_lookup=True over the 26 features, int32 [B_req, valency] ids in
  pinned host memory, the row pointers generated by the operator, and the
  26 pooled [B_req, 128] outputs copied back into pinned host memory."""

  def __init__(self, xse, wl, batch):
    ops = xse.ops
    self.resource = ops.CpuEmbeddingResource.empty(torch.cuda.current_device())
    engine = self.resource.engine
    for name, rows, combine, _, _, _, _, _ in wl.tables:
      engine.add_table(name, rows, combine, adopt=True)
      engine.register_feature(name, name)
    self.transform = ops.CpuEmbeddingLookupTransform(
        self.resource, wl.names, dense_lookup=True, embedding_dim=REF_DIM)
    self.sets = []
    calls = REF_BATCH // batch
    for v in range(REF_ROTATE):
      for c in range(calls):
        ids_l = []
        for t, (ids, _) in enumerate(wl.sets[v]):
          val = REF_VALENCY[t]
          buf = ops.PinnedBuffer((batch, val), np.int32)
          buf.array[:] = ids[c * batch * val:(c + 1) * batch * val].view(
              batch, val).cpu().numpy()
          ids_l.append(buf)
        self.sets.append(ids_l)
    self.h2d_bytes = sum(b.array.nbytes for b in self.sets[0])
    self.d2h_bytes = batch * len(REF_VOCAB) * REF_DIM * 4
    self.prepared = [ops.PreparedInputs(ids_l) for ids_l in self.sets]

  def step(self, i, stream=None):
    outs = self.transform.output_array()
    self.transform.run_prepared(self.prepared[i % len(self.prepared)], outs,
                                stream=stream)
    self.transform.free_outputs(outs)

  run = OperatorHostInputs.run

  def close(self):
    for lst in self.sets:
      for b in lst:
        b.close()
    self.transform.close()
    self.resource.close()


def measure_dlrm_lookup(xse, args, world, local):
  """The reference bundle's lookup workload: examples/s on the device
  (batch 16384), end to end through the dense-lookup operator at the
  published per-call batch of 128 with concurrent callers, CPU baseline and
  parity at N=1."""
  wl = DlrmLookupWorkload(xse, int(os.environ.get("RANK", "0")))
  for i in range(args.warmup):
    wl.step(i)
  wl.status.wait()
  ms, launches = timed_steps(wl.step, args.warmup, args.steps, world, local)
  wl.status.wait()
  pool_ms, pool_n, val_ms = kernel_timing(wl.engine, wl.step,
                                          args.warmup + args.steps,
                                          KERNEL_TIMING_LAUNCHES)
  wl.status.wait()
  examples = sum_over_ranks(REF_BATCH * args.steps, world)
  peak, peak_kind = measured_peaks()
  achieved = wl.bytes_per_step() / (pool_ms / 1000.0) / 1e9
  threads = args.lookup_threads
  host = DenseLookupHostInputs(xse, wl, REF_BATCH_REQ)
  host.run(2 * threads, threads)
  barrier(world, local)
  e_calls = 256
  e_ms = max_over_ranks(host.run(e_calls, threads), world)
  e_examples = sum_over_ranks(REF_BATCH_REQ * e_calls, world)
  h2d, d2h = host.h2d_bytes, host.d2h_bytes
  host.close()
  base = parity = None
  if world == 1 and not args.no_cpu_baseline:
    oracle = load_oracle()
    cores = oracle.host_cores()
    bags = []
    for t, (name, rows, _, _, _, _, _, _) in enumerate(wl.tables):
      ids, rp = wl.sets[0][t]
      bags.append(oracle.Bag(rows.cpu().numpy(), ids.cpu().numpy(),
                             rp.cpu().numpy(), None, "SUM", oracle.F32))
    oracle.embedding_bag_batch(bags, num_threads=cores)
    reps, t0 = 0, time.perf_counter()
    while True:
      oracle.embedding_bag_batch(bags, num_threads=cores)
      reps += 1
      el = time.perf_counter() - t0
      if el >= 3.0:
        break
    cpu = reps * REF_BATCH / el
    base = {"value": cpu, "unit": "examples/s", "cores": cores,
            "kind": "port", "per_core": cpu / cores,
            "sample": f"{reps} full batches of {REF_BATCH} examples (26 "
                      f"tables, 214 ids per example) in {el:.1f} s"}
    wl.step(0)
    torch.cuda.synchronize()
    wl.status.wait()
    parity = check_parity(wl.parity_items(0), 1024)
  result = {
      "metric": "DLRM lookup examples/sec", "value": examples / (ms / 1000.0),
      "unit": "examples/s", "n_gpus": world, "steps": args.steps,
      "ms_per_step": ms / args.steps, "dtype": "f32",
      "scaling": "weak",
      "config": {"workload": "dlrm_lookup: the reference DLRM bundle's "
                             "lookup -- 26 fp32 tables of its vocabulary "
                             "sizes x 128, valencies 1..100 (214 ids per "
                             "example), uniform int32 ids, dense_lookup "
                             "row pointers, SUM pooling",
                 "batch_per_gpu": REF_BATCH, "batch_per_call_e2e":
                     REF_BATCH_REQ},
      "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak,
                   "peak_kind": peak_kind, "unit": "GB/s",
                   "frac": achieved / peak,
                   "algorithmic_bytes_per_step": wl.bytes_per_step(),
                   "avg_launch_ms": pool_ms, "timed_launches": pool_n,
                   "traffic": None},
      "validation": validation_share(val_ms, ms / args.steps),
      "e2e": {"value": e_examples / (e_ms / 1000.0), "unit": "examples/s",
              "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
              "path": "CpuEmbeddingLookupTransform(dense_lookup=True) with "
                      f"int32 [{REF_BATCH_REQ}, valency] ids in pinned host "
                      f"memory; {threads} host threads issue calls "
                      "concurrently (one stream each); a step is one call"},
      "published_reference": {
          "value": REF_PUBLISHED, "unit": "examples/core-s",
          "where": "XSE C++ embedding kernel at B_req=128 on the "
                   "reference's host (docs/benchmarks/dlrm_serving.md:"
                   "240-244)"},
      "gpu_launches": launches,
      "cpu_baseline": base,
      "parity": parity,
  }
  wl.close()
  del wl
  torch.cuda.synchronize()
  torch.cuda.empty_cache()
  return result


# ---------------------------------------------------------------------------
# The reference arm.


def run_reference(args):
  """CPU restatement of the reference path on all host cores, on the same
  seeded inputs as the GPU arm (the counter RNG restated on the host), same
  metric and config; each step pools a bounded sample of the batch."""
  world = int(os.environ.get("WORLD_SIZE", "1"))
  rank = int(os.environ.get("RANK", "0"))
  if rank != 0:
    return
  oracle = load_oracle()
  cores = oracle.host_cores()
  weighted = [k < 4 for k in range(NUM_TABLES)]
  combine = ["SUM" if k < 4 else "MEAN" for k in range(NUM_TABLES)]
  tables = []
  for k in range(NUM_TABLES):
    bits, _, _ = oracle.synth_rows(oracle.BF16, SEED, k, 0, VOCAB, DIM)
    tables.append(bits)
  # The GPU arm's inputs: table k, variant v draws its ids (uniform) and
  # weights from stream k + 1000 v with fixed lengths of BAG.
  inputs = []
  for v in range(ROTATE):
    feats = []
    for k in range(NUM_TABLES):
      stream = k + 1000 * v
      ids = oracle.synth_ids(BATCH * BAG, VOCAB, SEED, stream)
      w = (oracle.synth_weights(BATCH * BAG, SEED, stream)
           if weighted[k] else None)
      feats.append((ids, w))
    inputs.append(feats)

  def make_bags(v, bags_per_table):
    out = []
    n = bags_per_table * BAG
    offsets = np.arange(bags_per_table + 1, dtype=np.int64) * BAG
    for k in range(NUM_TABLES):
      ids, w = inputs[v][k]
      out.append(oracle.Bag(tables[k], ids[:n], offsets,
                            None if w is None else w[:n], combine[k],
                            oracle.BF16))
    return out

  probe = make_bags(0, BATCH)
  t0 = time.perf_counter()
  oracle.embedding_bag_batch(probe, num_threads=cores)
  full = time.perf_counter() - t0
  budget = 120.0 / max(args.steps + args.warmup, 1)
  frac = min(1.0, budget / max(full, 1e-6))
  bags_per_step = max(64, int(BATCH * frac))
  sets = [make_bags(v, bags_per_step) for v in range(ROTATE)]
  for i in range(args.warmup):
    oracle.embedding_bag_batch(sets[i % ROTATE], num_threads=cores)
  t0 = time.perf_counter()
  for i in range(args.steps):
    oracle.embedding_bag_batch(sets[(args.warmup + i) % ROTATE],
                               num_threads=cores)
  el = time.perf_counter() - t0
  ids = args.steps * NUM_TABLES * bags_per_step * BAG
  value = ids / el
  sample = (f"{bags_per_step} of {BATCH} bags per table per step "
            f"({NUM_TABLES} tables, {BAG} ids per bag)")
  line = {
      "impl": "reference", "metric": "embedding-bag ids/sec",
      "value": value, "unit": "ids/s", "n_gpus": world,
      "steps": args.steps, "warmup": args.warmup,
      "ms_per_step": 1000.0 * el / max(args.steps, 1),
      "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
      "dtype": "bf16", "data": DATA,
      "config": multi_table_config(world, args.exchange),
      "cpu_baseline": {"value": value, "unit": "ids/s", "cores": cores,
                       "kind": "port", "sample": sample},
      "e2e": {"value": value, "unit": "ids/s", "h2d_bytes_per_step": 0,
              "d2h_bytes_per_step": 0},
  }
  print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Stand-alone workload runs.


def run_config(args, name):
  world, rank, local = init_distributed()
  torch.cuda.set_device(local)
  xse = load_package()
  clocks = ClockSampler(local)
  clocks.start()
  line = measure_config(xse, args, name, world, rank, local, args.max_rows)
  line["clocks"] = clocks.stop()
  line["vs_baseline"] = None
  if rank == 0:
    print(json.dumps(line), flush=True)
  if world > 1:
    dist.destroy_process_group()


def run_dlrm_only(args):
  """The DLRM forward alone, as its own JSON line."""
  world, rank, local = init_distributed()
  torch.cuda.set_device(local)
  xse = load_package()
  clocks = ClockSampler(local)
  clocks.start()
  result = measure_dlrm(xse, args, world, local)
  result["clocks"] = clocks.stop()
  result["warmup"] = args.warmup
  result["higher_is_better"] = True
  result["scaling"] = "weak"
  result["vs_baseline"] = None
  result["data"] = "synthetic (seeded counter RNG)"
  if rank == 0:
    print(json.dumps(result), flush=True)
  if world > 1:
    dist.destroy_process_group()


def run_dlrm_lookup_only(args):
  world, rank, local = init_distributed()
  torch.cuda.set_device(local)
  xse = load_package()
  clocks = ClockSampler(local)
  clocks.start()
  result = measure_dlrm_lookup(xse, args, world, local)
  result["clocks"] = clocks.stop()
  result["warmup"] = args.warmup
  result["higher_is_better"] = True
  result["vs_baseline"] = None
  result["data"] = "synthetic (seeded counter RNG, uniform ids)"
  if rank == 0:
    print(json.dumps(result), flush=True)
  if world > 1:
    dist.destroy_process_group()


def run_asset_load(args):
  """Host asset -> HBM upload rate of the table loader (one GPU): a
  `--asset-gib` fp32 table (dim 128) written as a `.bin` asset with its
  manifest, then loaded through xse_resource_load_sharded with one pageable
  cudaMemcpy per table and with the pinned double-buffered chunked upload;
  the file is in the page cache after it is written (the rate is memory ->
  HBM, not disk)."""
  import tempfile  # pylint: disable=import-outside-toplevel
  xse = load_package()
  torch.cuda.set_device(0)
  dim = 128
  rows = int(args.asset_gib * (1 << 30)) // (dim * 4)
  nbytes = rows * dim * 4
  with tempfile.TemporaryDirectory(prefix="xse_bench_assets_") as tmp:
    path = os.path.join(tmp, "big.bin")
    with open(path, "wb") as f:
      block = np.arange(1 << 20, dtype=np.float32)  # 4 MiB
      left = rows * dim
      while left > 0:
        n = min(left, block.size)
        f.write(block[:n].tobytes())
        left -= n
    manifest = os.path.join(tmp, "manifest.textproto")
    with open(manifest, "w", encoding="utf-8") as f:
      f.write(f'tables {{ name: "big" vocab_size: {rows} embedding_dim: '
              f'{dim} combine_mode: SUM }}\n'
              'feature_specs { name: "f" table: "big" }\n')
    assets = {"__jce_manifest__": manifest, "big": path}
    result = {}
    for label, chunk, placement in (("pageable", -1, None),
                                    ("chunked", 0, None),
                                    ("rowwise_quarter", 0, ("row", 4, 0))):
      times = []
      for _ in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = xse.ops.CpuEmbeddingResource.from_assets(
            assets, 0, placement=placement, chunk_bytes=chunk)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
        res.close()
      loaded = nbytes // 4 if placement else nbytes
      result[label] = {"seconds": min(times),
                       "GBps": loaded / min(times) / 1e9}
  line = {
      "metric": "table asset load GB/s (host file -> HBM)",
      "value": result["chunked"]["GBps"], "unit": "GB/s", "n_gpus": 1,
      "higher_is_better": True, "data": "synthetic fp32 table asset",
      "config": {"workload": f"asset_load: one fp32 table {rows} x {dim} "
                             f"({nbytes / 2**30:.2f} GiB), page-cached file",
                 "upload": "32 MiB pinned chunks filled by 8 pread "
                           "threads, "
                           "double-buffered"},
      "pageable_GBps": result["pageable"]["GBps"],
      "rowwise_quarter_GBps": result["rowwise_quarter"]["GBps"],
      "detail": result}
  print(json.dumps(line), flush=True)


EXTRAS = ("zipf_single", "sharded_tablewise", "int8_rowwise", "dlrm_forward",
          "dlrm_lookup")


def main():
  ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
  ap.add_argument("--gpus", type=int, default=1)
  ap.add_argument("--steps", type=int, default=200)
  ap.add_argument("--warmup", type=int, default=10)
  ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
  ap.add_argument("--e2e-steps", type=int, default=200)
  ap.add_argument("--e2e-threads", type=int, default=E2E_THREADS,
                  help="concurrent host callers of the operator in the e2e "
                       "run")
  ap.add_argument("--lookup-threads", type=int, default=4,
                  help="concurrent host callers of the dense-lookup operator "
                       "in dlrm_lookup's end-to-end run")
  ap.add_argument("--cpu-seconds", type=float, default=10.0)
  ap.add_argument("--no-cpu-baseline", action="store_true",
                  help="skip the CPU baselines and the parity checks")
  ap.add_argument("--exchange", default="peer",
                  choices=["a2a", "pipelined", "peer"],
                  help="N>1: one NCCL all-to-all after pooling, per-block "
                       "NCCL send/recv overlapped with the pooling, or "
                       "pooled rows stored into the owners' buffers over "
                       "NVLink by the pooling kernel")
  ap.add_argument("--dlrm-steps", type=int, default=40,
                  help="timed DLRM forward steps")
  ap.add_argument("--dlrm-max-rows", type=float, default=None,
                  help="cap the DLRM tables' rows (profiler captures)")
  ap.add_argument("--max-rows", type=float, default=None,
                  help="cap the tables' rows of a --workload config "
                       "(profiler captures)")
  ap.add_argument("--asset-gib", type=float, default=4.0,
                  help="--workload asset_load: size of the table asset")
  ap.add_argument("--extras", default=",".join(EXTRAS),
                  help="comma-separated workloads measured after the "
                       "headline in the default run ('none' for none)")
  ap.add_argument("--workload", default="multi_table",
                  choices=["multi_table", "dlrm", "dlrm_lookup",
                           "asset_load"] + sorted(CONFIGS),
                  help="multi_table (the headline line with every extra "
                       "workload), or one workload alone as its own line")
  args = ap.parse_args()
  args.warmup = max(args.warmup, MIN_WARMUP)
  if args.impl == "reference":
    run_reference(args)
    return
  if args.workload == "dlrm":
    run_dlrm_only(args)
    return
  if args.workload == "dlrm_lookup":
    run_dlrm_lookup_only(args)
    return
  if args.workload == "asset_load":
    run_asset_load(args)
    return
  if args.workload != "multi_table":
    run_config(args, args.workload)
    return
  extras = [] if args.extras in ("", "none") else args.extras.split(",")
  for name in extras:
    if name not in EXTRAS:
      raise SystemExit(f"unknown extra workload {name!r}")

  world, rank, local = init_distributed()
  torch.cuda.set_device(local)
  xse = load_package()
  clocks = ClockSampler(local)
  clocks.start()
  wl = Workload(xse, rank, world, args.exchange)

  # Warm-up (the engine's kernel tuner makes its choice on these: its trial
  # executions alternate the two pooling kernels, and the synchronize
  # below lets the first timed step read their timings).
  for i in range(args.warmup):
    wl.step(i)
  wl.finish()
  wl.check()
  elapsed_ms, launches = timed_steps(wl.step, args.warmup, args.steps, world,
                                     local, wl.finish)
  wl.check()
  first = args.warmup + args.steps
  pool_avg_ms, pool_n, val_ms = kernel_timing(wl.engine, wl.step, first,
                                              KERNEL_TIMING_LAUNCHES,
                                              wl.finish)
  wl.check()

  # End to end with host buffers: the operator at N=1, the sharded exchange
  # at N > 1.
  if world == 1:
    host = OperatorHostInputs(
        xse,
        [(spec.name, wl.tables[k], spec.combine, None, None, VOCAB, 0, 0)
         for k, spec in enumerate(wl.specs)],
        [[(fb.ids, fb.offsets, fb.weights) for fb in batch]
         for batch in wl.inputs], BATCH, DIM)
    host.run(3 * args.e2e_threads, args.e2e_threads)
    e2e_ms = host.run(args.e2e_steps, args.e2e_threads)
    e2e_steps = args.e2e_steps
    e2e_path = ("CpuEmbeddingLookupTransform (xse_lookup_transform_run, C "
                "ABI) over 8 features with pinned host inputs; H2D, "
                "validation, pooling and D2H of the outputs inside each "
                f"synchronous call; {args.e2e_threads} host threads issue "
                "calls concurrently (one stream each)")
    h2d, d2h = host.h2d_bytes, host.d2h_bytes
    host.close()
  else:
    sh = ShardedHostInputs(
        wl.run_exchange,
        [[(fb.ids, fb.offsets, fb.weights) for fb in batch]
         for batch in wl.inputs], BATCH // world * NUM_TABLES * world * DIM)
    e2e_steps = max(8, args.steps // 2)
    e2e_ms = timed_e2e(sh.step, e2e_steps, world, local)
    e2e_path = ("sharded exchange with host buffers: this rank's 8 tables' "
                "ids, offsets and weights (whole batch) copied from pinned "
                f"memory, pooling plus the {args.exchange} exchange, this "
                "rank's received pooled rows [B/N, 8N, 128] copied back, "
                "synchronous per step")
    h2d, d2h = sh.h2d_bytes, sh.d2h_bytes

  base = parity = None
  if world == 1 and not args.no_cpu_baseline:
    base = cpu_baseline(wl, args.cpu_seconds)
    v = first % ROTATE
    wl.step(v)
    torch.cuda.synchronize()
    wl.check()
    parity = check_parity(wl.parity_items(v), BATCH)
  # Per-rank spread of the pooling kernel's time (every rank takes part).
  pool_lo = min_over_ranks(pool_avg_ms, world)
  pool_hi = max_over_ranks(pool_avg_ms, world)
  ids_total = sum_over_ranks(wl.ids_per_step() * args.steps, world)
  value = ids_total / (elapsed_ms / 1000.0)
  e2e_ids = sum_over_ranks(wl.ids_per_step() * e2e_steps, world)
  e2e_value = e2e_ids / (e2e_ms / 1000.0)
  peak, peak_kind = measured_peaks()
  bytes_step = algorithmic_bytes_per_step()
  achieved = bytes_step / (pool_avg_ms / 1000.0) / 1e9
  wl.close()
  del wl
  torch.cuda.synchronize()
  torch.cuda.empty_cache()

  extra = {}
  for name in extras:
    if name == "dlrm_forward":
      extra[name] = measure_dlrm(xse, args, world, local)
    elif name == "dlrm_lookup":
      extra[name] = measure_dlrm_lookup(xse, args, world, local)
    else:
      extra[name] = measure_config(xse, args, name, world, rank, local)
  clock_info = clocks.stop()

  if rank == 0:
    line = {
        "metric": "embedding-bag ids/sec",
        "value": value,
        "unit": "ids/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": DATA,
        "config": multi_table_config(world, args.exchange),
        "hbm_gbs_algorithmic_step": bytes_step / (elapsed_ms / args.steps /
                                                  1000.0) / 1e9,
        "roofline": {
            "bound": "hbm",
            "kernel": "the pooling kernel the engine's tuner keeps for this "
                      "launch (PoolVecKernel<bf16, G=8, V=2, exact, wide> on "
                      "uniform ids over tables larger than L2), one launch "
                      "serving both weighting modes",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": POOL_DRAM_BYTES_PER_STEP if world == 1 else None,
            "traffic_source": "ncu dram__bytes_read.sum + "
                              "dram__bytes_write.sum of the pooling launch "
                              "on this workload (one GPU)",
            "algorithmic_bytes_per_launch": bytes_step,
            "avg_launch_ms": pool_avg_ms,
            "timed_launches": pool_n,
            "timing": "CUDA events around the pooling launch of each of "
                      f"{pool_n} steps run after the timed region",
        },
        "e2e": {
            "value": e2e_value,
            "unit": "ids/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "path": e2e_path,
        },
        "gpu_launches": launches,
        "ranks": {
            "step_ms": elapsed_ms / args.steps,
            "pool_ms_min": pool_lo,
            "pool_ms_max": pool_hi,
            "step_minus_slowest_pool_ms": elapsed_ms / args.steps - pool_hi,
            "note": "step = max over ranks of the timed region / steps; "
                    "pooling = each rank's CUDA-event mean over the "
                    "kernel-timing pass; the remainder is validation not "
                    "hidden under the previous step, the exchange's "
                    "synchronisation and launch gaps"},
        "validation": validation_share(val_ms, elapsed_ms / args.steps),
        "cpu_baseline": base,
        "parity": parity,
        "clocks": clock_info,
    }
    line.update(extra)
    print(json.dumps(line), flush=True)
  if world > 1:
    dist.destroy_process_group()


if __name__ == "__main__":
  main()
