"""CPU checks of the C ABI boundary: the library loads and exports every entry
point that include/*.h declares (no compute calls, no GPU needed)."""

import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
  names = set()
  for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
    with open(header, encoding="utf-8") as f:
      text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    for m in re.finditer(r"\b(xse_\w+)\s*\(", text):
      names.add(m.group(1))
  return names


def test_headers_declare_entry_points():
  names = declared_functions()
  assert "xse_engine_execute_batch" in names
  assert "xse_dot_interaction" in names
  assert len(names) >= 15


def test_library_exports_every_declared_symbol(xse):
  lib = ctypes.CDLL(xse._capi.LIB_PATH)
  missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
  assert not missing, missing


def test_bindings_cover_every_declared_symbol(xse):
  bound = set(xse._capi.SIGNATURES)
  assert declared_functions() <= bound, declared_functions() - bound


def test_abi_version_and_error_channel(xse):
  assert xse._capi.lib.xse_abi_version() == 1
  # A failing call without a GPU reports through xse_last_error.
  handle = ctypes.c_void_p()
  rc = xse._capi.lib.xse_status_create(0, ctypes.byref(handle))
  assert rc == xse._capi.INVALID_ARGUMENT
  assert "max_requests" in xse._capi.last_error()


def test_prepared_batch_holds_the_same_request_array(xse):
  """PreparedBatch converts its requests once; the array it hands the C ABI
  equals a fresh per-call conversion, and it still reads as the list."""
  import torch  # pylint: disable=import-outside-toplevel
  ids = torch.arange(10, dtype=torch.int64)
  offsets = torch.tensor([0, 4, 10], dtype=torch.int32)
  weights = torch.ones(10)
  out = torch.zeros(2, 3, 8)
  reqs = [xse.BagRequest(f"f{k}", ids, offsets, out[:, k, :],
                         weights if k == 1 else None, output_stride=24)
          for k in range(3)]
  prepared = xse.PreparedBatch(reqs)
  assert list(prepared) == reqs
  fresh, _ = xse.EmbeddingEngine._c_requests(reqs)  # pylint: disable=protected-access
  fields = [f for f, _ in xse._capi.BagRequest._fields_]  # pylint: disable=protected-access
  for k in range(3):
    for f in fields:
      assert getattr(prepared.array[k], f) == getattr(fresh[k], f), (k, f)
  assert prepared.array[2].output == out[:, 2, :].data_ptr()
  assert prepared.array[1].num_weights == 10 and prepared.array[0].weights is None
