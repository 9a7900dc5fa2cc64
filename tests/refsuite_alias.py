"""pytest plugin: the reference's own test suite imports ``crukx_sync``; this makes that name (and
its ``wire`` and ``codec`` modules) resolve to crukx_sync_b200 before the suite is collected, so
the reference's tests run unmodified against this package.  Loaded with ``-p refsuite_alias`` by
tests/test_gpu_reference_suite.py."""

import sys

import crukx_sync_b200
import crukx_sync_b200.codec
import crukx_sync_b200.wire

sys.modules["crukx_sync"] = crukx_sync_b200
sys.modules["crukx_sync.wire"] = crukx_sync_b200.wire
sys.modules["crukx_sync.codec"] = crukx_sync_b200.codec
