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
