"""Test configuration: the `gpu` marker, the package loader and fixtures."""

import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
  sys.path.insert(0, ROOT)

PACKAGE_DIR = os.path.join(ROOT, "xla-serving_b200")
PACKAGE_NAME = "xla_serving_b200"


def load_package():
  """Imports the engine package from its directory (its name has a hyphen)."""
  if PACKAGE_NAME in sys.modules:
    return sys.modules[PACKAGE_NAME]
  spec = importlib.util.spec_from_file_location(
      PACKAGE_NAME, os.path.join(PACKAGE_DIR, "__init__.py"),
      submodule_search_locations=[PACKAGE_DIR])
  module = importlib.util.module_from_spec(spec)
  sys.modules[PACKAGE_NAME] = module
  try:
    spec.loader.exec_module(module)
  except BaseException:
    del sys.modules[PACKAGE_NAME]
    raise
  return module


def pytest_configure(config):
  config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def gpu_available():
  try:
    import torch  # pylint: disable=import-outside-toplevel
    return torch.cuda.is_available()
  except ImportError:
    return False


def pytest_collection_modifyitems(config, items):
  del config
  if gpu_available():
    return
  skip = pytest.mark.skip(reason="no CUDA device")
  for item in items:
    if "gpu" in item.keywords:
      item.add_marker(skip)


@pytest.fixture(scope="session")
def xse():
  """The engine package (CUDA library loaded)."""
  return load_package()


@pytest.fixture(scope="session")
def golden():
  import json  # pylint: disable=import-outside-toplevel
  with open(os.path.join(ROOT, "tests", "golden", "known_answers.json"),
            encoding="utf-8") as f:
    return json.load(f)
