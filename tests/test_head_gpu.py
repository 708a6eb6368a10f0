"""The greedy head with its argmax keys folded into the tensor-core GEMV's epilogue, on one GPU
(a one-rank communicator): tests/head_worker.py in its own process."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_one_rank_head_matches_argmax():
    port = 29100 + os.getpid() % 500
    cmd = ["timeout", "-k", "30", "600", sys.executable, os.path.join(HERE, "head_worker.py"), str(port)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0 and "HEAD_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
