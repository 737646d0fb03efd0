"""CPU checks of the benchmark's arithmetic and report helpers: the
algorithmic bytes of the headline step (every id's row and id, the weights
of the weighted tables, int64 offsets, fp32 outputs), the kernels a sharded
step launches, the validation entry of the JSON line, single-process rank
reductions, and the multi-table config dict."""

import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
  spec = importlib.util.spec_from_file_location(
      "bench_under_test", os.path.join(ROOT, "bench.py"))
  module = importlib.util.module_from_spec(spec)
  spec.loader.exec_module(module)
  return module


def test_headline_algorithmic_bytes(bench):
  nnz = 8 * 8192 * 20
  want = (nnz * (256 + 8) + 4 * 8192 * 20 * 4 + 8193 * 8 * 8 +
          8192 * 8 * 128 * 4)
  assert bench.algorithmic_bytes_per_step() == want == 382_730_304


def test_exchange_launches(bench):
  assert bench.exchange_launches("peer", 1) == 2
  assert bench.exchange_launches("peer", 4) == 3  # + the flag barrier
  assert bench.exchange_launches("a2a", 2) == 3   # + the reorder
  assert bench.exchange_launches("pipelined", 4) == 9
  assert bench.exchange_launches("row", 2, chunks=4) == 8


def test_validation_share(bench):
  assert bench.validation_share(None, 0.07) is None
  v = bench.validation_share(0.0125, 0.0625)
  assert v["ms_per_step"] == 0.0125
  assert v["fraction_of_step"] == pytest.approx(0.2)


def test_single_rank_reductions(bench):
  assert bench.max_over_ranks(3.5, 1) == 3.5
  assert bench.min_over_ranks(3.5, 1) == 3.5
  assert bench.sum_over_ranks(7, 1) == 7


def test_multi_table_config(bench):
  cfg = bench.multi_table_config(4, "peer")
  assert cfg["global_batch"] == 8192 and cfg["tables_per_gpu"] == 8
  assert "workload" in cfg and "model" not in cfg
