"""Host side of expert parallelism, without a GPU:

* the per-rank plans: all eight slots (six routed, two shared) dealt round-robin over the ranks,
  every slot on exactly one rank, the exchange operators in place;
* the IPC handle exchange of fleet.ep.EpGroup over a two-rank gloo group with the library calls
  faked, and the peer table it writes;
* the arithmetic of the split: two gloo ranks each compute their slots of one MoE layer with the
  CPU oracle, exchange the slot rows (all_gather) and combine all eight in slot order; the result
  must equal the one-rank oracle bit for bit, as the kernel's exchange must.
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "fleet-amd-task_b200"))
sys.path.insert(0, str(ROOT))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_plans_deal_the_slots(world):
    from fleet import build_graph as B
    from fleet import mk
    from fleet.graph_plan import ep_slots
    from fleet.pack_weights import REAL_DIMS as d
    dealt = []
    for rank in range(world):
        plan, ops = B.dry_run(layers=4, ep=(rank, world))
        assert not plan.chain_violations()
        labels = [c.label for c in plan.calls]
        for l in range(1, 4):
            i13s, i13, i2 = labels.index(f"L{l}.w13s"), labels.index(f"L{l}.w13r"), labels.index(f"L{l}.w2_combine")
            assert i13s < i13 < i2
            gs, g, w2 = ops[i13s], ops[i13], ops[i2]
            assert gs["flags"] & mk.F_EP and g["flags"] & mk.F_EP and w2["flags"] & mk.F_EP
            assert (g["ips"][5], g["ips"][6], g["ips"][7]) == (rank, world, 0)
            assert (gs["ips"][5], gs["ips"][6], gs["ips"][7]) == (rank, world, d.TOPK)
            assert (w2["ips"][6], w2["ips"][7]) == (rank, world) and w2["ips"][8] == l - 1
            assert w2["ips"][5] == d.TOPK
            assert w2["ptrs"][mk.P["w2"]["PEERS"]] == "ep_peers" and mk.P["w2"]["OUT8"] not in w2["ptrs"]
        dealt += ep_slots(rank, world, d.N_SLOTS)
    # every slot on exactly one rank, and no rank more than one slot above another
    assert sorted(dealt) == list(range(d.N_SLOTS))
    counts = [len(ep_slots(r, world, d.N_SLOTS)) for r in range(world)]
    assert max(counts) - min(counts) <= 1


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from fleet import ep as E
    from fleet import mk
    base = 0x100000 * (rank + 1)
    mk.ep_alloc = lambda dev, n: base
    mk.ep_free = lambda p: None
    mk.ep_ipc_handle = lambda p: p.to_bytes(8, "little") * 8
    mk.ep_ipc_open = lambda dev, h: int.from_bytes(h[:8], "little") + 0x7000000000
    mk.ep_ipc_close = lambda p: None

    def all_gather(obj):
        objs = [None] * world
        dist.all_gather_object(objs, obj)
        return objs

    g = E.EpGroup(rank, world, 0, 8, 2048, 26, all_gather, table_device="cpu")
    t = mk.MkEpPeers.from_buffer_copy(bytes(g.table.numpy()))
    q.put((rank, [t.xch[r] for r in range(world)], t.nranks, t.rank, (t.n_layers, t.n_slots, t.hidden),
           g.slots(), g.xch_bytes))
    g.close()
    dist.destroy_process_group()


def test_ep_group_exchanges_handles_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29400 + os.getpid() % 500
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, xch, n, me, geom, slots, nbytes in res:
        assert (n, me) == (2, rank)
        assert geom == (26, 8, 2048) and nbytes == 2 * 26 * 8 * 1024 * 8
        assert slots == [s for s in range(8) if s % 2 == rank]
        for r in range(2):
            own = 0x100000 * (r + 1)
            assert xch[r] == (own if r == rank else own + 0x7000000000)


# ---- the split's arithmetic: oracle ranks over gloo against one rank

def _moe_inputs():
    from oracle.detmath import bf16
    from tests.ep_worker import small_dims
    d = small_dims()
    rng = np.random.default_rng(7)
    w = lambda *s: bf16((rng.standard_normal(s) * 0.05).astype(np.float32))  # noqa: E731
    return d, dict(x=bf16(rng.standard_normal(d.H).astype(np.float32)), w_norm=bf16(1 + 0.3 * rng.standard_normal(d.H)),
                   W_gate=w(d.E, d.H), W13=w(d.E_TOTAL, 2 * d.I_MOE, d.H), W2=w(d.E_TOTAL, d.H, d.I_MOE))


def _slot_rows(d, t, h, mask, slots):
    """The down-projection rows of the given slots (what a rank computes and sends)."""
    from oracle import numpy_ref as R
    out = {}
    for s in slots:
        e = int(mask[s])
        mid = R.linear(h, t["W13"][e])
        out[s] = R.linear(R.swiglu_act(mid, d.I_MOE), t["W2"][e])
    return out


def _oracle_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from fleet.graph_plan import ep_slots
    from oracle import numpy_ref as R
    d, t = _moe_inputs()
    h, logits, topk_w, routing, mask = R.moe_router_norm(t["x"], t["w_norm"], t["W_gate"], topk=d.TOPK,
                                                         n_experts=d.E, forced=tuple(range(d.E, d.E_TOTAL)))
    mine = _slot_rows(d, t, h, mask, ep_slots(rank, world, d.N_SLOTS))
    every = [None] * world
    dist.all_gather_object(every, mine)          # the exchange: every rank's slot rows
    out8 = np.full((d.N_SLOTS, d.H), np.nan, np.float32)
    for part in every:
        for s, row in part.items():
            assert np.isnan(out8[s]).all(), f"slot {s} computed twice"
            out8[s] = row
    q.put((rank, R.moe_combine(out8, topk_w, t["x"]), mask))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_split_matches_one_rank_over_gloo(world):
    from oracle import numpy_ref as R
    d, t = _moe_inputs()
    h, logits, topk_w, routing, mask = R.moe_router_norm(t["x"], t["w_norm"], t["W_gate"], topk=d.TOPK,
                                                         n_experts=d.E, forced=tuple(range(d.E, d.E_TOTAL)))
    rows = _slot_rows(d, t, h, mask, range(d.N_SLOTS))
    want = R.moe_combine(np.stack([rows[s] for s in range(d.N_SLOTS)]), topk_w, t["x"])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29900 + (os.getpid() + world) % 500
    ps = [ctx.Process(target=_oracle_rank, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=180) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, m in res:
        assert np.array_equal(m, mask)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"rank {rank} differs from one rank"
