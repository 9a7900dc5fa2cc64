"""The reference's own test suite (tests/test_roundtrip.py of crukx-sync), unmodified, against this
package: ``crukx_sync`` is aliased to ``crukx_sync_b200`` (tests/refsuite_alias.py) and the suite
runs in a child pytest.

The suite file is not part of this repository.  It is looked up beside the reference install at
``baseline/_ref/tests/test_roundtrip.py`` (or at the path in CRUKX_REF_SUITE); without it this test
is skipped.  Two tests of the suite exercise the reference's internals rather than its interface
and are deselected:
  * test_multi_slab_paths_and_slab_boundaries monkeypatches ``codec._SLAB``, the reference's slab
    size (this package has no slabs; slab-crossing tensors are covered by the golden case
    ``multislab`` and the 2^28/2^31-element parity tests);
  * test_triton_decoder_matches_torch_decoder switches the reference between its Triton and torch
    decoders (this package has one CUDA decoder).
"""

import os
import re
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
DESELECT = ["test_multi_slab_paths_and_slab_boundaries", "test_triton_decoder_matches_torch_decoder"]


def suite_path():
    return os.environ.get("CRUKX_REF_SUITE") or os.path.join(ROOT, "baseline", "_ref", "tests", "test_roundtrip.py")


def test_reference_suite_passes_against_this_package():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    path = suite_path()
    if not os.path.exists(path):
        pytest.skip(f"the reference's test suite is not at {path}")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([HERE, ROOT] + [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "refsuite_alias", "-p", "no:cacheprovider",
           "--rootdir", os.path.dirname(path), "-c", os.devnull, os.path.basename(path)]
    for name in DESELECT:
        cmd += ["--deselect", f"{os.path.basename(path)}::{name}"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900, cwd=os.path.dirname(path))
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    m = re.search(r"(\d+) passed", r.stdout)
    assert m and int(m.group(1)) >= 25, tail
    assert "failed" not in r.stdout.splitlines()[-1], tail
    print(r.stdout.splitlines()[-1])
