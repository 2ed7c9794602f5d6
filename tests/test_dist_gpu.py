"""Data parallelism on 2 GPUs: a step whose global batch is split over two
ranks (each one micro-batch; gradients all-reduced in several NCCL buckets
during backward, averaged inside the fused AdamW) equals a step on one GPU
that accumulates both micro-batches. Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_dp2_equals_single_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, HERE)
    import dist_step_worker as W
    from tinytrain_b200 import trainer as trn
    out = str(tmp_path / "dp.npz")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300", sys.executable, "-m",
                        "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr=127.0.0.1", "--master-port=29531",
                        os.path.join(HERE, "dist_step_worker.py"), out],
                       capture_output=True, text=True, env=env)
    if r.returncode != 0:
        lines = [ln for ln in (r.stdout + r.stderr).splitlines()
                 if "Error" in ln or "error" in ln or "Traceback" in ln]
        raise AssertionError("\n".join(lines[-30:]))
    dp = np.load(out)
    rng = np.random.default_rng(0)
    w = (rng.standard_normal(2_000_000) * 0.05).astype(np.float32)
    idx = rng.integers(0, W.CFG["vocab"], W.GLOBAL * W.T)
    tgt = rng.integers(0, W.CFG["vocab"], W.GLOBAL * W.T)
    torch.cuda.set_device(0)
    tr = trn.Trainer(W.CFG, seed=1, host_init=False)
    tr.set_params(w[:tr.n_params].copy())
    tr.set_optimizer(lr=1e-2, clip=1.0)
    loss, gn = tr.step(idx, tgt, W.B, W.T, W.GLOBAL // W.B, 1e-2)
    assert abs(float(dp["loss"]) - loss) <= 1e-5 * abs(loss)
    assert abs(float(dp["gn"]) - gn) <= 1e-4 * gn
    assert rel_err(dp["params"], tr.get_params()) < 1e-5
    tr.close()
