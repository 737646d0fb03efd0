"""Seeded synthetic workloads generated on the device.

Every value is a counter-based function of (seed, stream, index) computed by
the engine's synth kernels, so any table or id array can be regenerated
elsewhere. Shapes and value distributions follow the workloads the engine is
measured on:
  * single table: 1,000,000 x 64 fp32, batch 4096, bag lengths U[1,32],
    Zipf(1.05) ids, sum pooling;
  * multi-table: 8 bf16 tables 500,000 x 128, batch 8192, 20 ids per bag,
    uniform ids, per-id weights U(0,1); tables 0-3 weighted sum, 4-7 mean;
  * DLRM: 26 fp32 tables, dim 128, rows log-uniform in [1e4, 1e7], bag
    lengths U[1,100], Zipf(1.05) ids, sum pooling, batch 16384;
  * sharded: 64 bf16 tables 20,000,000 x 128, batch 65536, lengths U[1,64],
    Zipf(1.1);
  * int8 row-wise: 26 tables 10,000,000 x 256, batch 32768, lengths U[1,80],
    Zipf(1.05).
"""

import ctypes
import dataclasses
import math
from typing import List, Optional

import torch

from . import _capi as C
from .engine import stream_handle

# Multiplier of the Zipf rank -> row permutation; reduced to a value coprime
# with the table's row count by coprime_multiplier().
PERM_MUL = 2654435761
PERM_ADD = 40503


def coprime_multiplier(vocab, mul=PERM_MUL):
  m = mul % vocab
  if m == 0:
    m = 1
  while math.gcd(m, vocab) != 1:
    m += 1
  return m


def synth_table(dtype, vocab, dim, seed, table, device="cuda", row0=0,
                nrows=None, stream=None):
  """Rows [row0, row0+nrows) of synthetic table `table`.

  Returns (rows, scale, bias); scale and bias are None except for int8.
  """
  nrows = vocab - row0 if nrows is None else nrows
  tdt = {C.DT_F32: torch.float32, C.DT_BF16: torch.bfloat16,
         C.DT_I8_ROWWISE: torch.int8}[dtype]
  rows = torch.empty((nrows, dim), dtype=tdt, device=device)
  scale = bias = None
  if dtype == C.DT_I8_ROWWISE:
    scale = torch.empty(nrows, dtype=torch.float32, device=device)
    bias = torch.empty(nrows, dtype=torch.float32, device=device)
  C.check(C.lib.xse_synth_table(
      rows.data_ptr(), None if scale is None else scale.data_ptr(),
      None if bias is None else bias.data_ptr(), dtype, seed, table, row0,
      nrows, dim, stream_handle(stream)))
  return rows, scale, bias


def synth_lengths(n, lo, hi, seed, table, device="cuda", stream=None):
  out = torch.empty(n, dtype=torch.int64, device=device)
  C.check(C.lib.xse_synth_lengths(out.data_ptr(), n, lo, hi, seed, table,
                                  stream_handle(stream)))
  return out


def synth_ids(n, vocab, seed, table, zipf_alpha=0.0, index0=0, device="cuda",
              stream=None):
  out = torch.empty(n, dtype=torch.int64, device=device)
  mul = coprime_multiplier(vocab)
  C.check(C.lib.xse_synth_ids(out.data_ptr(), n, vocab, float(zipf_alpha),
                              mul, PERM_ADD % vocab, seed, table, index0,
                              stream_handle(stream)))
  return out


def synth_weights(n, seed, table, index0=0, device="cuda", stream=None):
  out = torch.empty(n, dtype=torch.float32, device=device)
  C.check(C.lib.xse_synth_weights(out.data_ptr(), n, seed, table, index0,
                                  stream_handle(stream)))
  return out


def offsets_from_lengths(lengths):
  """CSR offsets (int64, num_bags + 1) from bag lengths (stream-ordered)."""
  offsets = torch.zeros(lengths.numel() + 1, dtype=torch.int64,
                        device=lengths.device)
  torch.cumsum(lengths, 0, out=offsets[1:])
  return offsets


@dataclasses.dataclass
class TableSpec:
  name: str
  vocab: int
  dim: int
  dtype: int
  combine: str
  weighted: bool = False


@dataclasses.dataclass
class FeatureBatch:
  """One table's CSR batch on the device."""
  ids: torch.Tensor
  offsets: torch.Tensor
  weights: Optional[torch.Tensor]


def synth_batch(spec: TableSpec, table_index, batch, len_lo, len_hi, seed,
                zipf_alpha=0.0, variant=0, device="cuda"):
  """A CSR batch for one table. `variant` selects an independent draw
  (different counter ranges), used to rotate inputs between steps."""
  stream_table = table_index + 1000 * variant
  if len_lo == len_hi:
    lengths = torch.full((batch,), len_lo, dtype=torch.int64, device=device)
  else:
    lengths = synth_lengths(batch, len_lo, len_hi, seed, stream_table, device)
  offsets = offsets_from_lengths(lengths)
  nnz = int(offsets[-1].item())
  ids = synth_ids(nnz, spec.vocab, seed, stream_table, zipf_alpha,
                  device=device)
  weights = synth_weights(nnz, seed, stream_table,
                          device=device) if spec.weighted else None
  return FeatureBatch(ids, offsets, weights)


def log_uniform_rows(num_tables, lo, hi, seed):
  """Row counts log-uniform in [lo, hi], deterministic in seed."""
  g = torch.Generator().manual_seed(seed)
  u = torch.rand(num_tables, generator=g, dtype=torch.float64)
  return [int(round(math.exp(math.log(lo) + float(x) *
                             (math.log(hi) - math.log(lo))))) for x in u]


def multi_table_specs() -> List[TableSpec]:
  """8 bf16 tables 500,000 x 128: 0-3 weighted sum, 4-7 mean."""
  specs = []
  for t in range(8):
    specs.append(TableSpec(f"table_{t}", 500_000, 128, C.DT_BF16,
                           "SUM" if t < 4 else "MEAN", weighted=t < 4))
  return specs
