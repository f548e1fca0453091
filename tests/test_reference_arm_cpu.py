"""The benchmark's reference arm on CPU, launched as the round-end runs launch it.

``bench.py --impl reference`` times the reference's own CPU implementation of the workload
(its ``speccache/kernels/reference.py`` functions from the installed copy under
``baseline/_ref``, or the oracle port when that copy is missing, with the reason in the line).
Under torchrun with two ranks, rank 0 alone prints one JSON line and both ranks exit 0.
"""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import REPO


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(600)
def test_reference_arm_two_ranks_one_line():
    env = dict(os.environ, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "bench.py",
           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3",
           "--workload", "paged"]
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=540)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [json.loads(x) for x in proc.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, proc.stdout
    line = lines[0]
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    base = line["cpu_baseline"]
    installed = os.path.exists(os.path.join(REPO, "baseline", "_ref", "speccache", "kernels",
                                            "reference.py"))
    assert base["kind"] == ("reference" if installed else "port")
    if not installed:
        assert "reference_unavailable" in base
