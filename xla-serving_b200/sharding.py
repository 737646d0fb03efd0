"""Embedding tables sharded across the GPUs of one node, one process per GPU.

The reference engine keeps every table in one host's memory
(data/cpu_embedding/cc/cpu_embedding_engine.h:41-103); tables larger than one
GPU's HBM are split here in the two standard ways, with the pooled outputs
exchanged over NVLink by NCCL (through torch.distributed):

* Table-wise: table t lives on rank t mod W. The ids of a table are given to
  its owner for the whole batch (model-parallel input layout). Each rank pools
  its T_local tables for all B samples into blocks [W][B/W][T_local][D], block
  s holding the samples owned by rank s (samples [s B/W, (s+1) B/W)); an
  all-to-all returns every block to its owner, which ends with the blocks
  [B/W][T_q][D] of every source rank q (row k of block q is global table
  q + k W).
* Row-wise: every table's rows are split into W contiguous windows of the
  (permuted) row space; rank r holds rows [r V / W, (r+1) V / W) of each
  table and sees all ids. Ids outside the window are skipped by the pooling
  kernel, while bag lengths and weight sums still count every id, so the
  per-rank partial sums add up to the full bag. A reduce-scatter (sum) leaves
  rank r with recv[B/W][T][D] for its samples. Sums of partials differ from
  the single-table CSR-order sum by rounding only.

The exchanges are pipelined with the pooling: the table-wise path pools the
block for rank r+j, hands it to NCCL (send to r+j, receive from r-j, the
shifted pairwise schedule, deadlock-free) and pools the next block while it
is in flight; the row-wise path splits the batch into chunks and
reduce-scatters chunk c while chunk c+1 is pooled.

A bag request over samples [b0, b1) of a CSR batch is the same ids and
weights with the offsets slice [b0, b1] (absolute offsets, first entry may be
above zero, as the reference's EmbeddingBagInput allows,
data/cpu_embedding/cc/embedding_bag.h:66-72), so sample blocks need no copies.

When the input arrives data-parallel instead (each rank holds every table's
ids for its own sample block), IdsAllToAll moves each table's block to the
table's owner first: one packing launch (include/xse_shard.h) per rank and
NCCL all-to-alls of the extents, the rebased offsets, the ids and the
weights; the owner pools block s straight from source s's chunk.
"""

import ctypes
import dataclasses
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _capi as C
from .engine import (BagRequest, PreparedBatch, last_launch_count,
                     stream_handle)


@dataclasses.dataclass(frozen=True)
class ShardPlan:
  """Placement of tables, rows and samples over `world` ranks."""

  world: int
  rank: int

  def __post_init__(self):
    if self.world < 1 or not 0 <= self.rank < self.world:
      raise ValueError(f"bad rank {self.rank} of world {self.world}")

  def table_owner(self, table: int) -> int:
    return table % self.world

  def tables_of(self, rank: int, num_tables: int) -> List[int]:
    """Global indices of the tables rank `rank` holds (table-wise)."""
    return list(range(rank, num_tables, self.world))

  def row_window(self, vocab: int, rank: Optional[int] = None
                 ) -> Tuple[int, int]:
    """Rows [begin, end) of a `vocab`-row table held by `rank` (row-wise)."""
    r = self.rank if rank is None else rank
    return vocab * r // self.world, vocab * (r + 1) // self.world

  def block_size(self, batch: int) -> int:
    if batch % self.world:
      raise ValueError(
          f"batch {batch} must split evenly over {self.world} ranks")
    return batch // self.world

  def sample_block(self, batch: int, rank: int) -> Tuple[int, int]:
    """Samples [begin, end) owned by `rank`."""
    n = self.block_size(batch)
    return rank * n, (rank + 1) * n


def slice_request(req: BagRequest, bag_begin: int, bag_end: int,
                  output: torch.Tensor, output_stride: int = 0) -> BagRequest:
  """The request for bags [bag_begin, bag_end) of `req`, writing `output`."""
  return BagRequest(req.feature_name, req.ids,
                    req.offsets[bag_begin:bag_end + 1], output, req.weights,
                    output_stride)


Pooler = Callable[[Sequence[BagRequest]], None]


class engine_pooler:  # pylint: disable=invalid-name
  """A pooler running each group on `engine`. With a `status` the groups run
  asynchronously (no host wait per group; read the result with
  status.wait() after the exchange). `launches` counts the kernels the
  groups launched."""

  def __init__(self, engine, status=None, fused=False):
    self.engine = engine
    self.status = status
    self.fused = fused
    self.launches = 0

  def __call__(self, reqs):
    self.engine.execute_batch(reqs, status=self.status, fused=self.fused)
    self.launches += last_launch_count()


class DevicePointer:
  """A raw device address standing in for a tensor as a bag request output
  (a peer's buffer mapped into this process)."""

  def __init__(self, address: int):
    self.address = address

  def data_ptr(self) -> int:
    return self.address


class _CudaArray:
  """__cuda_array_interface__ over raw fp32 device memory, for torch views."""

  def __init__(self, address, shape):
    self.__cuda_array_interface__ = {
        "shape": tuple(shape), "typestr": "<f4", "data": (address, False),
        "version": 3, "strides": None}


class PeerGroup:
  """Buffers of all ranks mapped into every rank, plus a stream-ordered flag
  barrier (include/xse_peer.h). Handles travel over torch.distributed."""

  def __init__(self, plan: ShardPlan, nbytes: int, device: int, group=None):
    self.plan = plan
    self.nbytes = nbytes
    self._handle = ctypes.c_void_p()
    mine = C.IpcHandle()
    C.check(C.lib.xse_peer_group_create(device, plan.world, plan.rank, nbytes,
                                        ctypes.byref(self._handle),
                                        ctypes.byref(mine)))
    gathered = [None] * plan.world
    dist.all_gather_object(gathered, bytes(mine.bytes), group=group)
    handles = (C.IpcHandle * plan.world)()
    for q, raw in enumerate(gathered):
      ctypes.memmove(handles[q].bytes, raw, len(raw))
    C.check(C.lib.xse_peer_group_connect(self._handle, handles, plan.world))
    self.group = group

  def address(self, rank: int) -> int:
    return C.lib.xse_peer_group_buffer(self._handle, rank)

  def local_view(self, offset_bytes: int, shape) -> torch.Tensor:
    """fp32 tensor over this rank's buffer."""
    return torch.as_tensor(
        _CudaArray(self.address(self.plan.rank) + offset_bytes, shape),
        device="cuda")

  def barrier(self, stream=None, spin_limit=0):
    C.check(C.lib.xse_peer_group_barrier(self._handle, spin_limit,
                                         stream_handle(stream)))

  def check(self, stream=None):
    C.check(C.lib.xse_peer_group_check(self._handle, stream_handle(stream)))

  def close(self):
    if self._handle:
      torch.cuda.synchronize()
      dist.barrier(group=self.group)  # every rank is done with the others'
      C.lib.xse_peer_group_destroy(self._handle)
      self._handle = ctypes.c_void_p()


CsrFeature = Tuple[str, torch.Tensor, torch.Tensor, Optional[torch.Tensor]]


def _index_type(t: torch.Tensor) -> int:
  if t.dtype == torch.int64:
    return C.INDEX_I64
  if t.dtype == torch.int32:
    return C.INDEX_I32
  raise TypeError(f"ids and offsets must be int32 or int64, got {t.dtype}")


class CsrPacker:
  """The packing kernels of include/xse_shard.h over device tensors. A job
  is (ids, offsets, weights, dst_ids, dst_offsets, dst_weights, dst_base):
  bags [0, len(offsets) - 1) of the source, their id range copied to dst_ids
  (and weights to dst_weights when both are given) and the offsets rebased
  to start at dst_base written to dst_offsets (int64)."""

  @staticmethod
  def _segments(jobs, with_dst):
    segs = (C.CsrSegment * max(len(jobs), 1))()
    for k, (ids, offsets, weights, d_ids, d_offs, d_w, base) in enumerate(
        jobs):
      g = segs[k]
      g.ids = ids.data_ptr() if ids.numel() else None
      g.offsets = offsets.data_ptr()
      g.weights = None if weights is None else weights.data_ptr()
      g.num_ids = ids.numel()
      g.num_bags = offsets.numel() - 1
      g.ids_type = _index_type(ids)
      g.offsets_type = _index_type(offsets)
      if with_dst:
        g.dst_ids = d_ids.data_ptr() if d_ids.numel() else None
        g.dst_offsets = d_offs.data_ptr()
        g.dst_weights = (None if d_w is None or weights is None
                         else d_w.data_ptr())
        g.dst_base = base
    return segs

  def extents(self, jobs, stream=None) -> torch.Tensor:
    """int64 device tensor: each job's id count, -1 for a bad range."""
    out = torch.empty(len(jobs), dtype=torch.int64, device="cuda")
    if jobs:
      C.check(C.lib.xse_csr_extents(self._segments(jobs, False), len(jobs),
                                    out.data_ptr(), stream_handle(stream)))
    return out

  def pack(self, jobs, stream=None):
    if jobs:
      C.check(C.lib.xse_csr_pack(self._segments(jobs, True), len(jobs),
                                 stream_handle(stream)))


class IdsAllToAll:
  """Data-parallel input -> the table-wise layout.

  run(features): features[t] = (feature name, ids, offsets, weights) of
  global table t for this rank's sample block (offsets: B/W + 1 absolute
  entries; the same weighting per table on every rank). Returns blocks,
  blocks[s][k] = (name, ids, offsets, weights) of local table k (global
  table rank + k W) for the samples of rank s: offsets are B/W + 1 int64
  entries into source s's received chunk `ids` -- what
  TablewiseExchange.schedule(blocks=...) takes.

  Steps: the extents of the W x T_q slices (one launch), an all-to-all of
  them and one device->host read (the sizes NCCL needs), one packing launch
  that writes, per destination, its tables' id ranges back to back with
  rebased offsets, then all-to-alls of the offsets, the ids and (if any
  table is weighted) the weights.
  """

  def __init__(self, plan: ShardPlan, batch: int, num_tables: int,
               device=None, group=None, packer=None):
    self.plan = plan
    self.batch = batch
    self.num_tables = num_tables
    self.block = plan.block_size(batch)
    self.device = device
    self.group = group
    self.packer = CsrPacker() if packer is None else packer
    w = plan.world
    self.counts = [len(plan.tables_of(q, num_tables)) for q in range(w)]
    self.local = plan.tables_of(plan.rank, num_tables)
    # Send order: destination-major, each destination's tables in order.
    self.order = [t for q in range(w) for t in plan.tables_of(q, num_tables)]
    self.bytes_last = 0  # bytes this rank sent in the last run()

  def run(self, features: Sequence[CsrFeature]):
    w, nb = self.plan.world, self.block
    if len(features) != self.num_tables:
      raise ValueError(f"expected {self.num_tables} features, got "
                       f"{len(features)}")
    for name, _, offsets, _ in features:
      if offsets.numel() != nb + 1:
        raise ValueError(f"feature {name}: {offsets.numel()} row pointers, "
                         f"the sample block needs {nb + 1}")
    id_dtype = features[0][1].dtype
    if any(f[1].dtype != id_dtype for f in features):
      raise TypeError("all features' ids must share one dtype")
    weighted = [f[3] is not None for f in features]
    any_w = any(weighted)
    jobs_src = [(features[t][1], features[t][2], features[t][3])
                for t in self.order]
    ext = self.packer.extents([j + (None, None, None, 0) for j in jobs_src])
    n_local = len(self.local)
    recv_ext = torch.empty(w * n_local, dtype=torch.int64, device=ext.device)
    if w > 1:
      dist.all_to_all_single(recv_ext, ext, output_split_sizes=[n_local] * w,
                             input_split_sizes=self.counts, group=self.group)
    else:
      recv_ext.copy_(ext)
    host = torch.cat([ext, recv_ext]).cpu().tolist()
    send_ext, recv_list = host[:len(self.order)], host[len(self.order):]
    for t, e in zip(self.order, send_ext):
      if e < 0:
        raise C.XseError(C.INVALID_ARGUMENT,
                         f"feature {features[t][0]}: row pointers outside "
                         "the ids (negative, decreasing or past the end)")
    # Positions: each destination's chunk holds its tables back to back.
    bases, send_sizes, j = [], [], 0
    for q in range(w):
      at = 0
      for _ in range(self.counts[q]):
        bases.append(at)
        at += send_ext[j]
        j += 1
      send_sizes.append(at)
    recv_sizes = [sum(recv_list[s * n_local:(s + 1) * n_local])
                  for s in range(w)]
    dev = ext.device
    send_ids = torch.empty(sum(send_sizes), dtype=id_dtype, device=dev)
    send_offs = torch.empty((len(self.order), nb + 1), dtype=torch.int64,
                            device=dev)
    send_w = (torch.empty(sum(send_sizes), dtype=torch.float32, device=dev)
              if any_w else None)
    jobs, start, j = [], 0, 0
    for q in range(w):
      for _ in range(self.counts[q]):
        t = self.order[j]
        lo, hi = start + bases[j], start + bases[j] + send_ext[j]
        jobs.append(jobs_src[j] + (
            send_ids[lo:hi], send_offs[j],
            None if send_w is None else send_w[lo:hi], bases[j]))
        j += 1
      start += send_sizes[q]
    self.packer.pack(jobs)
    recv_ids = torch.empty(sum(recv_sizes), dtype=id_dtype, device=dev)
    recv_offs = torch.empty((w, n_local, nb + 1), dtype=torch.int64,
                            device=dev)
    recv_w = (torch.empty(sum(recv_sizes), dtype=torch.float32, device=dev)
              if any_w else None)
    if w > 1:
      dist.all_to_all_single(
          recv_offs.view(-1), send_offs.view(-1),
          output_split_sizes=[n_local * (nb + 1)] * w,
          input_split_sizes=[c * (nb + 1) for c in self.counts],
          group=self.group)
      dist.all_to_all_single(recv_ids, send_ids, output_split_sizes=recv_sizes,
                             input_split_sizes=send_sizes, group=self.group)
      if any_w:
        dist.all_to_all_single(recv_w, send_w, output_split_sizes=recv_sizes,
                               input_split_sizes=send_sizes, group=self.group)
    else:
      recv_offs.view(-1).copy_(send_offs.view(-1))
      recv_ids.copy_(send_ids)
      if any_w:
        recv_w.copy_(send_w)
    esize = send_ids.element_size()
    self.bytes_last = (sum(send_sizes) * (esize + (4 if any_w else 0)) +
                       send_offs.numel() * 8)
    blocks, start = [], 0
    for s in range(w):
      end = start + recv_sizes[s]
      chunk = recv_ids[start:end]
      wchunk = None if recv_w is None else recv_w[start:end]
      blocks.append([
          (features[t][0], chunk, recv_offs[s, k],
           wchunk if weighted[t] else None)
          for k, t in enumerate(self.local)])
      start = end
    return blocks


MODES = ("a2a", "pipelined", "peer")
# Receive slots of the peer exchange: a step may overwrite a slot once the
# barrier of the step after its previous use has passed on every rank, so
# three slots let one step's barrier overlap the next step's pooling.
PEER_SLOTS = 3


class TablewiseExchange:
  """Pools this rank's tables for the whole batch and returns each sample
  block to its owning rank.

  features (to schedule()): (feature name, ids, offsets, weights) of the
  local tables, in local table order, each over the whole batch.
  pool: runs a group of bag requests on the current stream
  (engine_pooler(engine, status) on the GPU).
  After run(), recv_from(q) is [B/W, T_q, D]: the pooled rows of rank q's
  tables (global tables q, q + W, ...) for this rank's samples.

  Modes:
    a2a: one group of whole-batch requests into send, then one NCCL
      all-to-all.
    pipelined: a group per destination block, each handed to NCCL
      send/recv (shifted pairwise schedule) while the next is pooled.
    peer: one group whose requests write every block straight into its
      owner's receive buffer over NVLink (CUDA IPC mappings), then one flag
      barrier (on a side stream); receive buffers rotate over PEER_SLOTS
      slots so a step's stores never overwrite rows still being read.
  """

  def __init__(self, plan: ShardPlan, batch: int, num_tables: int, dim: int,
               pool: Pooler, device=None, group=None, mode="a2a"):
    if mode not in MODES:
      raise ValueError(f"unknown exchange mode {mode!r}")
    self.plan = plan
    self.batch = batch
    self.num_tables = num_tables
    self.dim = dim
    self.pool = pool
    self.group = group
    self.mode = mode
    self.block = plan.block_size(batch)
    w = plan.world
    self.counts = [len(plan.tables_of(q, num_tables)) for q in range(w)]
    self.num_local = self.counts[plan.rank]
    self.recv_sizes = [self.block * c * dim for c in self.counts]
    self.recv_offsets = [sum(self.recv_sizes[:q]) for q in range(w)]
    total = self.block * num_tables * dim
    self.peers = None
    self.send = None
    self._slot = 0
    self._step = -1
    if mode == "peer" and w > 1:
      dev = torch.cuda.current_device() if device is None else (
          torch.device(device).index or torch.cuda.current_device())
      self.peers = PeerGroup(plan, PEER_SLOTS * total * 4, dev, group)
      self._slots = [self.peers.local_view(s * total * 4, (total,))
                     for s in range(PEER_SLOTS)]
      self._side = torch.cuda.Stream()
      self._done = [None] * PEER_SLOTS
    else:
      self.send = torch.empty((w, self.block, self.num_local, dim),
                              dtype=torch.float32, device=device)
      self._slots = [torch.empty(total, dtype=torch.float32, device=device)]

  @property
  def recv(self) -> torch.Tensor:
    return self._slots[self._slot]

  def recv_from(self, q: int, slot: Optional[int] = None) -> torch.Tensor:
    buf = self._slots[self._slot if slot is None else slot]
    at = self.recv_offsets[q]
    return buf[at:at + self.recv_sizes[q]].view(self.block, self.counts[q],
                                                self.dim)

  def sample_major(self, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The received rows as [B/W, T, D] in global table order."""
    if out is None:
      out = torch.empty((self.block, self.num_tables, self.dim),
                        dtype=torch.float32, device=self.recv.device)
    for q in range(self.plan.world):
      out[:, q::self.plan.world, :] = self.recv_from(q)
    return out

  def block_requests(self, features, dest: int, out, blocks=None):
    """Requests pooling the samples of rank `dest` into out, a [B/W, T_local,
    D] tensor or the DevicePointer of one: slices of the whole-batch
    `features`, or `blocks[dest]` (IdsAllToAll.run) as they are."""
    if blocks is not None:
      b0, b1, features = 0, self.block, blocks[dest]
    else:
      b0, b1 = self.plan.sample_block(self.batch, dest)
    row = self.num_local * self.dim
    reqs = []
    for k, (name, ids, offsets, weights) in enumerate(features):
      base = BagRequest(name, ids, offsets, None, weights)
      if isinstance(out, DevicePointer):
        dst = DevicePointer(out.address + 4 * k * self.dim)
      else:
        dst = out[:, k, :]
      reqs.append(slice_request(base, b0, b1, dst, row))
    return reqs

  def schedule(self, features=None, blocks=None):
    """The request groups of one exchange, built once and reused by run()
    (with `blocks` from IdsAllToAll.run, built again for every step's
    blocks).

    a2a: [(None, requests writing send)] (send [W][B/W][T_local][D] is
    [B][T_local][D] in sample order). pipelined: [(dest, requests)] for
    rank+1, rank+2, ..., then the own block pooled straight into recv.
    peer: one group per receive slot, each writing every rank's slot.
    Each group is a PreparedBatch (converted to the C request array once).
    """
    return [(key, PreparedBatch(reqs))
            for key, reqs in self._groups(features, blocks)]

  def _groups(self, features, blocks):
    w, r = self.plan.world, self.plan.rank
    local = features if blocks is None else blocks[r]
    if len(local) != self.num_local or (blocks is not None and
                                        len(blocks) != w):
      raise ValueError(f"rank {self.plan.rank} holds {self.num_local} tables, "
                       f"got {len(local)} features")
    if w == 1:
      return [(r, self.block_requests(features, r, self.recv_from(r),
                                      blocks))]
    if self.mode == "a2a":
      if blocks is not None:
        reqs = []
        for dest in range(w):
          reqs += self.block_requests(None, dest, self.send[dest], blocks)
        return [(None, reqs)]
      whole = self.send.view(self.batch, self.num_local, self.dim)
      reqs = [BagRequest(name, ids, offsets, whole[:, k, :], weights,
                         self.num_local * self.dim)
              for k, (name, ids, offsets, weights) in enumerate(features)]
      return [(None, reqs)]
    if self.mode == "pipelined":
      steps = []
      for j in range(1, w):
        dest = (r + j) % w
        steps.append((dest, self.block_requests(features, dest,
                                                self.send[dest], blocks)))
      steps.append((r, self.block_requests(features, r, self.recv_from(r),
                                           blocks)))
      return steps
    total = self.block * self.num_tables * self.dim
    groups = []
    for slot in range(PEER_SLOTS):
      reqs = []
      for dest in range(w):
        # Rank dest's slot holds [q][B/W][T_q][D]; this rank writes block r.
        at = 4 * (slot * total + self.recv_offsets[r])
        reqs += self.block_requests(
            features, dest, DevicePointer(self.peers.address(dest) + at),
            blocks)
      groups.append((slot, reqs))
    return groups

  def run(self, steps, wait=True):
    """Pools and exchanges the groups of schedule(). With wait (default) the
    current stream is ordered after the exchange on return (recv is ready
    for work queued on it). Peer mode with wait=False leaves the barrier on
    a side stream so the next step's pooling overlaps it; call ready()
    before reading recv. Either way the rows of a step must be consumed
    (their readers queued) before the next run()."""
    w, r = self.plan.world, self.plan.rank
    if w == 1:
      for _, reqs in steps:
        self.pool(reqs)
      return self.recv
    if self.mode == "a2a":
      self.pool(steps[0][1])
      send_size = self.block * self.num_local * self.dim
      dist.all_to_all_single(self.recv, self.send.view(-1),
                             output_split_sizes=self.recv_sizes,
                             input_split_sizes=[send_size] * w,
                             group=self.group)
      return self.recv
    if self.mode == "pipelined":
      works = []
      for j, (dest, reqs) in enumerate(steps):
        self.pool(reqs)
        if dest != r:
          src = (r - (j + 1)) % w
          ops = [dist.P2POp(dist.isend, self.send[dest], dest, self.group),
                 dist.P2POp(dist.irecv, self.recv_from(src), src, self.group)]
          works.extend(dist.batch_isend_irecv(ops))
      for work in works:
        work.wait()
      return self.recv
    i = self._step + 1
    slot = i % PEER_SLOTS
    main = torch.cuda.current_stream()
    # Step i overwrites the slot of step i - PEER_SLOTS on every rank. Each
    # rank queued that step's readers before its own pooling of step
    # i - PEER_SLOTS + 1, which the barrier of that step waited for.
    prev = self._done[(i - PEER_SLOTS + 1) % PEER_SLOTS]
    if i >= PEER_SLOTS - 1 and prev is not None:
      main.wait_event(prev)
    self.pool(steps[slot][1])
    pooled = torch.cuda.Event()
    pooled.record(main)
    self._side.wait_event(pooled)
    self.peers.barrier(stream=self._side)
    done = torch.cuda.Event()
    done.record(self._side)
    self._done[slot] = done
    self._step = i
    self._slot = slot
    if wait:
      main.wait_event(done)
    return self.recv

  def ready(self, stream=None):
    """Orders `stream` (the current one by default) after the last
    exchange's barrier."""
    if self.peers is not None and self._done[self._slot] is not None:
      (stream or torch.cuda.current_stream()).wait_event(
          self._done[self._slot])

  def check(self):
    """Raises if a peer barrier gave up waiting (peer mode)."""
    if self.peers is not None:
      self.peers.check()

  def close(self):
    if self.peers is not None:
      self._slots = []
      self.peers.close()
      self.peers = None


class RowwiseExchange:
  """Pools every table against this rank's row windows into partial sums
  and reduce-scatters them so that each rank ends with its samples' full
  pooled rows: recv [B/W, T, D].

  features: (feature name, ids, offsets, weights) per table over the whole
  batch (every rank sees all ids).
  chunks: the batch is pooled and reduce-scattered in this many pieces
  (block size divisible by it); chunk c of every rank's block is pooled
  together, so each reduce-scatter moves a [W][B/(W chunks)][T][D] piece.
  """

  def __init__(self, plan: ShardPlan, batch: int, num_tables: int, dim: int,
               pool: Pooler, chunks: int = 1, device=None, group=None):
    self.plan = plan
    self.batch = batch
    self.num_tables = num_tables
    self.dim = dim
    self.pool = pool
    self.group = group
    self.block = plan.block_size(batch)
    if chunks < 1 or self.block % chunks:
      raise ValueError(f"block of {self.block} samples does not split into "
                       f"{chunks} chunks")
    self.chunks = chunks
    self.piece = self.block // chunks
    self.recv = torch.empty((self.block, num_tables, dim),
                            dtype=torch.float32, device=device)
    if plan.world == 1:  # nothing to reduce: pool straight into recv
      self.partial = self.recv.view(chunks, 1, self.piece, num_tables, dim)
    else:
      self.partial = torch.empty((chunks, plan.world, self.piece, num_tables,
                                  dim), dtype=torch.float32, device=device)

  def chunk_requests(self, features, c: int) -> List[BagRequest]:
    reqs = []
    for s in range(self.plan.world):
      b0 = s * self.block + c * self.piece
      out = self.partial[c, s]
      for k, (name, ids, offsets, weights) in enumerate(features):
        base = BagRequest(name, ids, offsets, None, weights)
        reqs.append(slice_request(base, b0, b0 + self.piece, out[:, k, :],
                                  self.num_tables * self.dim))
    return reqs

  def schedule(self, features) -> List[List[BagRequest]]:
    """One PreparedBatch of requests per chunk, reused by run()."""
    return [PreparedBatch(self.chunk_requests(features, c))
            for c in range(self.chunks)]

  def run(self, steps):
    works = []
    for c, reqs in enumerate(steps):
      self.pool(reqs)
      out = self.recv[c * self.piece:(c + 1) * self.piece]
      if self.plan.world == 1:
        continue
      works.append(dist.reduce_scatter_tensor(
          out.view(-1), self.partial[c].view(-1), group=self.group,
          async_op=True))
    for work in works:
      work.wait()
    return self.recv


# ---------------------------------------------------------------------------
# The C ABI's sharded execution (include/xse_shard.h): the schedules above,
# run by the engine's C++ host code over its own NCCL communicator.

SHARD_MODES = {"peer": C.SHARD_TABLE_PEER, "a2a": C.SHARD_TABLE_A2A,
               "pipelined": C.SHARD_TABLE_PIPELINED, "row": C.SHARD_ROW}


class ShardComm:
  """The engine's NCCL communicator over the ranks of `group` (the default
  torch.distributed group): rank 0 draws the NCCL unique id through the C
  ABI and the id reaches every rank over torch.distributed."""

  def __init__(self, device: int, plan: ShardPlan, group=None):
    self.plan = plan
    self._handle = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(C.SHARD_ID_BYTES)
    if plan.rank == 0:
      C.check(C.lib.xse_shard_unique_id(uid))
    if plan.world > 1:
      box = [bytes(uid.raw)]
      dist.broadcast_object_list(box, src=0, group=group)
      uid = ctypes.create_string_buffer(box[0], C.SHARD_ID_BYTES)
    C.check(C.lib.xse_shard_comm_create(device, plan.world, plan.rank, uid,
                                        ctypes.byref(self._handle)))

  @property
  def handle(self):
    return self._handle

  def abort(self):
    if self._handle:
      C.check(C.lib.xse_shard_comm_abort(self._handle))

  def close(self):
    if self._handle:
      C.lib.xse_shard_comm_destroy(self._handle)
      self._handle = ctypes.c_void_p()


class ShardedExchange:
  """One sharded step per run() through xse_shard_exchange_run.

  mode: "peer", "a2a", "pipelined" (table-wise: global table t on rank
  t mod W; features are this rank's tables in local order) or "row"
  (every table's rows split over the ranks; features are all tables).
  features: (feature name, ids, offsets, weights) over the whole batch.
  run() returns this rank's pooled rows [B/W, T, D] (sample-major, global
  table order) as a view of the exchange's output slot, valid until the
  next run().
  """

  def __init__(self, engine, comm: ShardComm, mode: str, num_tables: int,
               dim: int, batch: int, chunks: int = 1, spin_limit: int = 0):
    self.comm = comm
    self.mode = mode
    self.plan = comm.plan
    self.num_tables = num_tables
    self.dim = dim
    self.batch = batch
    self.block = self.plan.block_size(batch)
    p = C.ShardPlanStruct(mode=SHARD_MODES[mode], num_tables=num_tables,
                          dim=dim, chunks=chunks, batch=batch,
                          spin_limit=spin_limit)
    self._handle = ctypes.c_void_p()
    C.check(C.lib.xse_shard_exchange_create(engine.handle, comm.handle,
                                            ctypes.byref(p),
                                            ctypes.byref(self._handle)))
    self.recv = None
    self._views = {}  # output slot address -> tensor view

  def prepare(self, features: Sequence[CsrFeature]) -> PreparedBatch:
    """The C request array of one step's features, built once."""
    return PreparedBatch([BagRequest(name, ids, offsets, None, weights)
                          for name, ids, offsets, weights in features])

  def run(self, prepared, stream=None, defer=False) -> torch.Tensor:
    if not isinstance(prepared, PreparedBatch):
      prepared = self.prepare(prepared)
    out = ctypes.c_void_p()
    C.check(C.lib.xse_shard_exchange_run(
        self._handle, prepared.array, len(prepared),
        C.SHARD_DEFER_WAIT if defer else 0, stream_handle(stream),
        ctypes.byref(out)))
    view = self._views.get(out.value)
    if view is None:
      shape = (self.block, self.num_tables, self.dim)
      view = torch.as_tensor(_CudaArray(out.value, shape), device="cuda")
      self._views[out.value] = view
    self.recv = view
    return view

  def ready(self, stream=None):
    C.check(C.lib.xse_shard_exchange_ready(self._handle,
                                           stream_handle(stream)))

  def check(self, stream=None):
    C.check(C.lib.xse_shard_exchange_check(self._handle,
                                           stream_handle(stream)))

  def close(self):
    if self._handle:
      torch.cuda.synchronize()
      if self.plan.world > 1 and dist.is_initialized():
        dist.barrier()  # every rank is done with the others' slots
      C.lib.xse_shard_exchange_destroy(self._handle)
      self._handle = ctypes.c_void_p()
