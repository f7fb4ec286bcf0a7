"""Test bootstrap.

* Pins the corpus n-gram order to 2 (``SUFFIX_HYBRID_INDEX_N``) before any
  test module constructs a proposer, so short fixtures resolve regardless of
  file order.  Production keeps the default order 8.
* Registers the ``gpu`` marker: tests that need a B200 are marked
  ``@pytest.mark.gpu`` and are run with ``-m gpu`` on a GPU host; everything
  else runs on CPU with ``-m "not gpu"``.
"""
import os
import sys

os.environ.setdefault("SUFFIX_HYBRID_INDEX_N", "2")
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running CPU test")
