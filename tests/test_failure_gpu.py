"""Failure paths on the device, none of which faults, traps or hangs a GPU.

- Bounded device waits: ttk_selftest_wait_timeout runs the mbarrier wait
  that every GEMM and attention pipeline uses on a barrier nothing arrives
  on, with a 5 ms limit. The kernel gives up, records the wait site in the
  device status word and returns; the context stays usable (a GEMM runs and
  checks out afterwards).
- The NCCL watchdog (2 GPUs): a rank leaves between steps; the other rank's
  next step fails within the collective deadline with the communicator
  aborted, later steps are refused, and the GPU still runs a fresh step.
  NVLS is off (NCCL_NVLS_ENABLE=0). Skipped with fewer than 2 GPUs.
"""
import json
import os
import subprocess
import sys
import time

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_bounded_wait_expires_and_reports_site(cuda):
    from tinytrain_b200 import _ttk
    _ttk.device_status()  # clear
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.time()
    _ttk.call("ttk_selftest_wait_timeout", 77, 5_000_000, stream)
    st = _ttk.device_status()  # synchronizes
    assert time.time() - t0 < 2.0
    assert st & 1, st
    assert (st >> 8) & 0xFF == 77, hex(st)
    # the context is intact: a GEMM runs and is right
    g = torch.Generator(device=cuda).manual_seed(3)
    A = torch.rand(256, 192, device=cuda, generator=g)
    B = torch.rand(192, 320, device=cuda, generator=g)
    C = torch.empty(256, 320, device=cuda)
    _ttk.call("ttk_gemm", 0, 0, 1, 256, 320, 192, 1.0, A.data_ptr(), 192, 0, B.data_ptr(), 320,
              0, 0.0, C.data_ptr(), 320, 0, None, 0, stream)
    torch.cuda.synchronize()
    assert rel_err(C.cpu().numpy(), (A.double() @ B.double()).cpu().numpy()) < 1e-4
    assert _ttk.device_status() == 0


def test_bounded_wait_rejects_bad_limits(cuda):
    from tinytrain_b200 import _ttk
    for site, lim in ((300, 1000), (1, 0), (1, 3_000_000_000)):
        with pytest.raises(_ttk.TtkError):
            _ttk.call("ttk_selftest_wait_timeout", site, lim, None)


def test_peer_leaves_watchdog_aborts(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "leave.json")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "180", sys.executable, "-m",
                        "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr=127.0.0.1", "--master-port=29533",
                        os.path.join(HERE, "dist_leave_worker.py"), out],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    res = json.load(open(out))
    assert res["error"] and ("did not complete" in res["error"] or
                             "asynchronous error" in res["error"]), res
    assert res["took"] < 60.0, res
    assert res["refused"] and "aborted" in res["refused"], res
    assert np.isfinite(res["loss_after"]) and res["status"] == 0, res
