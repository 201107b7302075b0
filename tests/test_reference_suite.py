"""The reference's own scheduler-side connector tests, unmodified, with this package's connector in place of NIXL.

lean-vLLM's tests/test_kv_transfer_scheduler.py drives its Scheduler and LLMEngine step loop through whatever
CONNECTORS["NixlConnector"] names: what the decode side admits, waits for and frees, what the prefill side holds,
hands over and releases, and the metrics of each. Run in a subprocess with tests/kvx_reference_swap.py loaded,
every one of those engines gets CudaIpcConnectorScheduler, and the file must pass as it does for the reference's.
Nothing is written into the checkout (no bytecode, no pytest cache). Skipped where no reference checkout is present
(REFERENCE_ROOT)."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE_ROOT = os.path.abspath(os.environ.get("REFERENCE_ROOT", os.path.join(ROOT, "..", "reference")))
if not os.path.isfile(os.path.join(REFERENCE_ROOT, "tests", "test_kv_transfer_scheduler.py")):
    pytest.skip("no lean-vLLM reference checkout with its tests", allow_module_level=True)


def test_the_reference_s_scheduler_tests_pass_with_this_connector(tmp_path):
    report = tmp_path / "made"
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([REFERENCE_ROOT, ROOT, os.path.join(ROOT, "tests")]),
               PYTHONDONTWRITEBYTECODE="1", KVX_SWAP_REPORT=str(report))
    run = subprocess.run(
        [sys.executable, "-m", "pytest", os.path.join(REFERENCE_ROOT, "tests", "test_kv_transfer_scheduler.py"),
         "-p", "kvx_reference_swap", "-p", "no:cacheprovider", "-q"],
        cwd=tmp_path, env=env, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout[-4000:] + run.stderr[-2000:]
    assert " passed" in run.stdout and "failed" not in run.stdout
    assert int(report.read_text()) >= 20  # the engines those tests built ran this package's scheduler half
