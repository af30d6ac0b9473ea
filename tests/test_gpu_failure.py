"""Failure detection without a GPU fault: a tensor-parallel rank that stops taking
part makes the other rank's bounded wait for its rows run out; that rank's call
returns B2_E_DEVICE (about a second later) instead of hanging, and its context
can still be destroyed. Rank 1 launches nothing, so both ranks can share one GPU;
NVLS is not involved (plain peer stores over CUDA IPC)."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_rank_that_leaves_makes_the_other_time_out(tmp_path):
    import torch
    ngpu = torch.cuda.device_count()
    port = str(_free_port())
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs, outs = [], []
    for r in range(2):
        out = tmp_path / f"r{r}.json"
        outs.append(out)
        dev = r if ngpu >= 2 else 0
        procs.append(subprocess.Popen([sys.executable, str(HERE / "tp_leave_worker.py"), str(r), "2", port, str(dev),
                                       str(out)], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=300)[0].decode(errors="replace"))
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
    for p, log in zip(procs, logs):
        assert p.returncode == 0, log[-3000:]
    r0 = json.loads(outs[0].read_text())
    assert r0["code"] == -8, r0                     # B2_E_DEVICE: the bounded wait ran out
    assert 0.5 < r0["seconds"] < 60, r0
    assert r0["device_err"] == 1                    # B2_DEV_ERR_TIMEOUT in the step state
    assert r0["destroyed"]
