"""GPU tests of the table asset loader's upload and placement
(xse_resource_load_sharded): tables read from `.bin` assets through pinned
staging chunks (many chunks, uneven slices, several fill threads), the
pageable single-copy path, and the table-wise / row-wise placements of a
sharded job. Every loaded row is read back through one-id bags (a SUM bag of
one id is the row itself: fp32 rows exactly, bf16 widened exactly, int8
rows dequantised) and compared with the oracle, bit for bit for fp32 and
bf16, within the int8 tolerance of the parity helpers for int8 rows; rows
outside a row-wise window pool to zero."""

import numpy as np
import pytest
import torch

from oracle import oracle
from parity_helpers import assert_pooled, expect_pool

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops(xse):
  return xse.ops


def make_tables(rng):
  f32 = rng.uniform(-1, 1, (1001, 24)).astype(np.float32)
  bits = (rng.uniform(-1, 1, (777, 40)).astype(np.float32).view(np.uint32)
          >> 16).astype(np.uint16)
  q = rng.integers(-127, 128, (613, 48)).astype(np.int8)
  sc = rng.uniform(1e-3, 1e-2, 613).astype(np.float32)
  bi = rng.uniform(-.1, .1, 613).astype(np.float32)
  return {"a": f32, "b": bits, "c": (q, sc, bi), "d": f32[:97, :8].copy(),
          "e": bits[:5, :16].copy()}


SPECS = [{"name": f"f{t}", "table_name": t} for t in "abcde"]
KIND = {"a": oracle.F32, "b": oracle.BF16, "c": oracle.I8_ROWWISE,
        "d": oracle.F32, "e": oracle.BF16}


def every_row(xse, engine, feature, vocab, dim):
  """Pools bag b = [id b] for every id: the table's rows as the engine sees
  them (zero rows outside a shard window)."""
  ids = torch.arange(vocab, dtype=torch.int64, device="cuda")
  offsets = torch.arange(vocab + 1, dtype=torch.int64, device="cuda")
  out = torch.empty((vocab, dim), device="cuda")
  engine.execute_batch([xse.BagRequest(feature, ids, offsets, out)])
  return out.cpu().numpy()


def want_rows(data, t, lo=None, hi=None):
  kind = KIND[t]
  if kind == oracle.I8_ROWWISE:
    q, sc, bi = data
    vocab = q.shape[0]
    rows, bound = expect_pool(q, kind, np.arange(vocab), np.arange(vocab + 1),
                              None, "SUM", sc, bi)
  else:
    vocab = data.shape[0]
    rows, bound = expect_pool(data, kind, np.arange(vocab),
                              np.arange(vocab + 1), None, "SUM")
  if lo is not None:
    rows = rows.copy()
    rows[:lo] = 0.0
    rows[hi:] = 0.0
  return rows, bound


def shape_of(data):
  return data[0].shape if isinstance(data, tuple) else data.shape


@pytest.mark.parametrize("chunk_bytes,threads", [(4096, 3), (1000, 1),
                                                 (-1, 0), (0, 0)])
def test_upload_paths(xse, ops, chunk_bytes, threads):
  rng = np.random.default_rng(21)
  tables = make_tables(rng)
  res = ops.CpuEmbeddingResource(tables, {t: "SUM" for t in tables}, SPECS,
                                 upload_threads=threads,
                                 chunk_bytes=chunk_bytes)
  for t, data in tables.items():
    vocab, dim = shape_of(data)
    assert_pooled(every_row(xse, res.engine, f"f{t}", vocab, dim),
                   want_rows(data, t), f"table {t}")
  res.close()


def test_tablewise_placement(xse, ops):
  rng = np.random.default_rng(22)
  tables = make_tables(rng)
  res = ops.CpuEmbeddingResource(tables, {t: "SUM" for t in tables}, SPECS,
                                 placement=("table", 3, 1), chunk_bytes=2048)
  for i, (t, data) in enumerate(tables.items()):
    vocab, dim = shape_of(data)
    assert res.get_embedding_dim(f"f{t}") == dim  # known for every feature
    if i % 3 == 1:
      assert_pooled(every_row(xse, res.engine, f"f{t}", vocab, dim),
                     want_rows(data, t), f"table {t}")
    else:
      with pytest.raises(xse.XseError) as e:
        every_row(xse, res.engine, f"f{t}", vocab, dim)
      assert e.value.code == xse._capi.NOT_FOUND
  res.close()


@pytest.mark.parametrize("rank", [0, 2])
def test_rowwise_placement(xse, ops, rank):
  rng = np.random.default_rng(23)
  tables = make_tables(rng)
  res = ops.CpuEmbeddingResource(tables, {t: "SUM" for t in tables}, SPECS,
                                 placement=("row", 3, rank), chunk_bytes=3000,
                                 upload_threads=2)
  for t, data in tables.items():
    vocab, dim = shape_of(data)
    lo, hi = vocab * rank // 3, vocab * (rank + 1) // 3
    info = res.engine.table_info(t)
    assert (info.row_begin, info.row_end, info.vocab) == (lo, hi, vocab)
    assert_pooled(every_row(xse, res.engine, f"f{t}", vocab, dim),
                   want_rows(data, t, lo, hi), f"table {t} rows {lo}-{hi}")
  res.close()


def test_bad_placement(xse, ops):
  tables = {"a": np.ones((4, 2), np.float32)}
  with pytest.raises(ValueError):
    ops.CpuEmbeddingResource(tables, {"a": "SUM"}, [], placement=("x", 2, 0))
  with pytest.raises(xse.XseError) as e:
    ops.CpuEmbeddingResource(tables, {"a": "SUM"}, [],
                             placement=("row", 2, 2))
  assert e.value.code == xse._capi.INVALID_ARGUMENT
  assert "Bad placement" in e.value.message
