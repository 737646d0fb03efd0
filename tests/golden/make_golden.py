"""Generates tests/golden/numpy_lookup.npz from the reference's own code.

The reference's DLRM benchmark keeps a numpy restatement of what its CPU
preprocessor computes, `embedding_lookup_numpy` and `embedding_lookup_stacked`
(examples/dlrm_benchmark/common.py, openxla/xla-serving). That module imports
grpc, JAX and generated protos at the top, none of which are importable here,
so this script extracts just those two functions from the source with `ast`
and runs them on seeded inputs. The resulting fixture pins the oracle (and,
through it, the CUDA path) to the reference's own lookup on dense-lookup SUM
bags, within fp32 summation-order tolerance.

It also records an addition-order case (values +-1e20, 31 + 6 ids) following
data/cpu_embedding/cc/embedding_bag_test.cc:296-343, whose expected output is
the strict CSR-order fp32 sum computed here with numpy float32 scalars.

Run from the repository root (needs the reference checkout, read only):
  python tests/golden/make_golden.py /path/to/reference
"""

import ast
import os
import sys

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)),
                   "numpy_lookup.npz")


def load_reference_functions(reference_root):
  path = os.path.join(reference_root, "examples", "dlrm_benchmark",
                      "common.py")
  with open(path, encoding="utf-8") as f:
    tree = ast.parse(f.read(), filename=path)
  wanted = {"embedding_lookup_numpy", "embedding_lookup_stacked",
            "_sparse_names"}
  body = [node for node in tree.body
          if isinstance(node, ast.FunctionDef) and node.name in wanted]
  found = {node.name for node in body}
  if "_sparse_names" not in found:
    # Older layouts name features '0'..'T-1'; supply the same convention.
    body.append(ast.parse(
        "def _sparse_names(n):\n  return [str(i) for i in range(n)]\n"
    ).body[0])
  missing = wanted - found - {"_sparse_names"}
  if missing:
    raise RuntimeError(f"functions not found in {path}: {sorted(missing)}")
  module = ast.Module(
      body=[ast.ImportFrom(module="__future__",
                           names=[ast.alias(name="annotations")], level=0)]
      + body,
      type_ignores=[])
  ast.fix_missing_locations(module)
  import functools  # pylint: disable=import-outside-toplevel
  import typing  # pylint: disable=import-outside-toplevel
  namespace = {"np": np, "functools": functools}
  namespace.update({"Sequence": typing.Sequence, "Mapping": typing.Mapping})
  exec(compile(module, path, "exec"), namespace)  # pylint: disable=exec-used
  return namespace["embedding_lookup_numpy"], namespace[
      "embedding_lookup_stacked"]


def addition_order_case():
  rows, dim = 4, 128
  values = np.array([1.0e20, 1.25, -1.0e20, 0.33333334], dtype=np.float32)
  table = np.zeros((rows, dim), dtype=np.float32)
  for r in range(rows):
    for c in range(dim):
      table[r, c] = np.float32(values[r]) + np.float32(c % 3) * np.float32(
          0.03125)
  ids = np.array([i % rows for i in range(37)], dtype=np.int64)
  offsets = np.array([0, 31, 37], dtype=np.int32)
  out = np.zeros((2, dim), dtype=np.float32)
  for b in range(2):
    acc = np.zeros(dim, dtype=np.float32)
    for p in range(offsets[b], offsets[b + 1]):
      acc = (acc + table[ids[p]]).astype(np.float32)
    out[b] = acc
  return table, ids, offsets, out


def main():
  if len(sys.argv) != 2:
    sys.exit(f"usage: {sys.argv[0]} REFERENCE_ROOT (the xla-serving source "
             "tree holding examples/dlrm_benchmark/common.py)")
  reference_root = sys.argv[1]
  lookup, stacked = load_reference_functions(reference_root)
  rng = np.random.default_rng(20260101)
  num_tables = 6
  batch = 64
  vocabs = [97, 1000, 5, 512, 33, 777]
  dims = [16, 8, 4, 16, 3, 12]
  valencies = [1, 3, 7, 20, 2, 33]
  tables = [rng.uniform(-0.05, 0.05, size=(v, d)).astype(np.float32)
            for v, d in zip(vocabs, dims)]
  features = {str(i): rng.integers(0, vocabs[i], size=(batch, valencies[i]),
                                   dtype=np.int64)
              for i in range(num_tables)}
  per_feature = lookup(tables, features)
  # The stacked variant needs one common dim: cross-check it on the dim-16
  # tables.
  same_dim = [i for i in range(num_tables) if dims[i] == 16]
  stacked_out = stacked([tables[i] for i in same_dim],
                        {str(k): features[str(i)]
                         for k, i in enumerate(same_dim)})
  for k, i in enumerate(same_dim):
    np.testing.assert_array_equal(per_feature[str(i)], stacked_out[:, k, :])

  order_table, order_ids, order_offsets, order_out = addition_order_case()
  arrays = {
      "num_tables": np.array(num_tables),
      "order_table": order_table,
      "order_ids": order_ids,
      "order_offsets": order_offsets,
      "order_out": order_out,
  }
  for i in range(num_tables):
    arrays[f"table_{i}"] = tables[i]
    arrays[f"ids_{i}"] = features[str(i)]
    arrays[f"out_{i}"] = per_feature[str(i)]
  np.savez_compressed(OUT, **arrays)
  print(f"wrote {OUT}")


if __name__ == "__main__":
  main()
