"""One rank of an expert-parallel decode run (launched by tests/test_gpu_ep.py through
torch.distributed.run): builds the same small model on every rank with fleet.ep.EpGroup, runs
greedy iterations in one launch, then a second launch of more iterations (the exchange tags carry
over launches), and writes this rank's tokens, route log and final residual to <out>/rank<r>.npz.
An odd MoE-layer count (the default: 4 layers, 3 MoE layers) checks that the exchange words of
one token's last MoE layer and the next token's first are not confused. Exit code 0 on success."""
import argparse
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "fleet-amd-task_b200"))


def small_dims():
    from fleet.pack_weights import Dims
    return Dims(H=256, NH=4, D_N=32, D_R=16, D_V=32, D_C=64, V=1024, L=4, I_DENSE=384, I_MOE=64, E=8, TOPK=2,
                N_SHARED=2)


def build(dims, layers, iters, n_past, seed, ep, device):
    import torch
    from fleet import build_graph as B
    from fleet.capture import make_capture
    from fleet.pack_weights import synthetic_packed
    s_max = n_past + 1 + iters
    packed = synthetic_packed(dims, layers=layers, head=True, seed=seed, device=device, random_norms=True)
    capture = make_capture(dims, layers, s_max, n_past, seed=seed + 1, device=device)
    prompt = torch.randint(0, dims.V, (n_past + 1,), generator=torch.Generator().manual_seed(seed + 2))
    meta = B.make_meta(torch, s_max, prompt.tolist(), n_past + 1, device=device)
    mpk, host, plan = B.build(packed, capture, meta, dims=dims, s_max=s_max, layers=layers, head=True, ep=ep,
                              wait_timeout_s=5.0)
    return mpk, host, meta, plan


def run(out, layers=4, iters=4, n_past=40, seed=0, second=3):
    import numpy as np
    import torch
    import torch.distributed as dist
    from fleet.ep import EpGroup
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))

    def all_gather(obj):
        objs = [None] * world
        dist.all_gather_object(objs, obj)
        return objs

    dims = small_dims()
    ep = EpGroup(rank, world, local, dims.N_SLOTS, dims.H, dims.L - 1, all_gather)
    mpk, host, meta, plan = build(dims, layers, iters + second, n_past, seed, ep, f"cuda:{local}")
    mpk.compile()
    dist.barrier()
    mpk.step = n_past - 1
    mpk.launch(iters)
    mpk.launch(second)
    torch.cuda.synchronize()
    st = mpk.status(raise_on_error=False)
    tokens = meta["tokens"][0].cpu().numpy()
    x_res = host["x_res"].view(torch.int16).cpu().numpy()
    np.savez(Path(out) / f"rank{rank}.npz", tokens=tokens, x_res=x_res, error=st["error"],
             route_log=host["route_log"].cpu().numpy())
    dist.barrier()          # every peer is done writing into this rank's buffers
    mpk.kernel.close()
    ep.close()
    dist.barrier()
    dist.destroy_process_group()
    return st["error"]


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--iters", type=int, default=4)
    a = ap.parse_args()
    sys.exit(1 if run(a.out, a.layers, a.iters) else 0)
