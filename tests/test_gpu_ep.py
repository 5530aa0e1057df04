"""Expert parallelism on 2, 4 and 8 GPUs of one node: every rank's greedy tokens, route log and
final residual must equal the one-GPU run's bit for bit (the combine adds the eight slots in slot
order on every rank, whichever rank computed them). The ranks run as child processes over two
launches (4 then 3 iterations of a 4-layer model, 3 MoE layers); skipped when the node has fewer
GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def one_gpu_reference():
    sys.path.insert(0, str(Path(__file__).resolve().parent))
    import ep_worker
    dims = ep_worker.small_dims()
    mpk, host, meta, plan = ep_worker.build(dims, 4, 7, 40, 0, None, "cuda:0")
    mpk.compile()
    mpk.step = 39
    mpk.launch(4)
    mpk.launch(3)
    torch.cuda.synchronize()
    assert mpk.status()["error"] == 0
    out = (meta["tokens"][0].cpu().numpy(), host["x_res"].view(torch.int16).cpu().numpy(),
           host["route_log"].cpu().numpy())
    mpk.kernel.close()
    return out


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_matches_one_gpu(tmp_path, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "500", sys.executable, "-m", "torch.distributed.run", "--standalone", "--nnodes=1",
           f"--nproc-per-node={world}", str(ROOT / "tests" / "ep_worker.py"), "--out", str(tmp_path)]
    r = subprocess.run(cmd, env=env, timeout=600, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    tokens, x_res, route_log = one_gpu_reference()
    for rank in range(world):
        got = np.load(tmp_path / f"rank{rank}.npz")
        assert int(got["error"]) == 0
        assert np.array_equal(got["tokens"], tokens), (rank, got["tokens"][38:], tokens[38:])
        assert np.array_equal(got["route_log"], route_log), rank
        assert np.array_equal(got["x_res"], x_res), rank
