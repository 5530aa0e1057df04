"""Expert parallelism on two GPUs of one node: every rank's greedy tokens and final residual must
equal the one-GPU run's bit for bit (the combine adds the eight slots in slot order on every rank,
whichever rank computed them). Runs the ranks as child processes; skipped below two GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep2_matches_one_gpu(tmp_path):
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    import ep_worker
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--nnodes=1", "--nproc-per-node=2",
           str(ROOT / "tests" / "ep_worker.py"), "--out", str(tmp_path)]
    r = subprocess.run(cmd, env=env, timeout=600, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    # the one-GPU run of the same model
    dims = ep_worker.small_dims()
    mpk, host, meta, plan = ep_worker.build(dims, 4, 4, 40, 0, None, "cuda:0")
    mpk.compile()
    meta["step"].fill_(39)
    mpk()
    torch.cuda.synchronize()
    assert mpk.status()["error"] == 0
    tokens = meta["tokens"][0].cpu().numpy()
    x_res = host["x_res"].view(torch.int16).cpu().numpy()
    mpk.kernel.close()
    for rank in range(2):
        got = np.load(tmp_path / f"rank{rank}.npz")
        assert int(got["error"]) == 0
        assert np.array_equal(got["tokens"], tokens), (rank, got["tokens"][38:], tokens[38:])
        assert np.array_equal(got["x_res"], x_res), rank
