"""Expert parallelism over the ranks of one node (one process per GPU), by slot.

Every rank runs the whole decode graph: attention, the dense layer 0, the embedding, the head,
the router and the shared experts are replicated (the router is deterministic, so all ranks route
alike). Every rank holds every expert's weights (31 GB in all, far below one GPU's 180 GB), so the
six routed slots of a token are dealt round-robin: rank r of N computes the routed slots s with
s mod N = r, whatever experts the router picked, and the ranks stay balanced at batch 1 (sharding
by expert id leaves a rank idle whenever the top-6 experts cluster on another). Each
down-projection task stores its rows of its rank's routed slots into the same rows of every
peer's exchange buffer, adds one to the peer's counter for (layer, task), waits until every
peer's same task has done the same, and adds the eight slots in slot order, so the result is the
one-GPU result bit for bit.

The exchange buffers are plain device memory from the library (cudaMalloc), mapped into the peers
with CUDA IPC; no multicast object is involved. Handles travel over the process group."""
import ctypes

from fleet import mk
from fleet.graph_plan import EP_PEERS_WORDS, ep_slots  # noqa: F401


class DeviceBuffer:
    """A device pointer with the tensor-like surface the operator builders read."""

    def __init__(self, ptr, shape, dtype_bytes, name):
        self.ptr, self.shape, self.dtype_bytes, self.name = ptr, tuple(shape), dtype_bytes, name

    def data_ptr(self):
        return self.ptr

    def numel(self):
        n = 1
        for s in self.shape:
            n *= s
        return n

    def dim(self):
        return len(self.shape)


class EpGroup:
    """This rank's exchange buffers, its peers' (opened through IPC) and the device peer table.

    n_slots, H: the out8 rows; n_layers: MoE layers (one arrival counter each). all_gather(obj)
    -> list of every rank's obj (torch.distributed.all_gather_object on the node's group)."""

    def __init__(self, rank, world, device, n_slots, H, n_layers, all_gather, table_device=None):
        import torch

        assert 1 <= world <= mk.EP_MAX_RANKS
        self.rank, self.world, self.device = rank, world, device
        self.n_slots, self.H, self.n_layers = n_slots, H, n_layers
        self.out8_bytes = 2 * n_slots * H * 2           # two layer-parity halves, BF16
        self.ctr_bytes = max(16, n_layers * mk.EP_MAX_TASKS * 4)   # [layers][tasks] counters
        self.out8_ptr = mk.ep_alloc(device, self.out8_bytes)
        self.ctr_ptr = mk.ep_alloc(device, self.ctr_bytes)
        handles = all_gather((mk.ep_ipc_handle(self.out8_ptr), mk.ep_ipc_handle(self.ctr_ptr)))
        self.peer_out8, self.peer_ctr, self.opened = [], [], []
        for r, (ho, hc) in enumerate(handles):
            if r == rank:
                self.peer_out8.append(self.out8_ptr)
                self.peer_ctr.append(self.ctr_ptr)
            else:
                po, pc = mk.ep_ipc_open(device, ho), mk.ep_ipc_open(device, hc)
                self.opened += [po, pc]
                self.peer_out8.append(po)
                self.peer_ctr.append(pc)
        table = mk.MkEpPeers()
        for r in range(world):
            table.out8[r] = self.peer_out8[r]
            table.counter[r] = self.peer_ctr[r]
        table.nranks, table.rank = world, rank
        raw = bytes(ctypes.string_at(ctypes.addressof(table), ctypes.sizeof(table)))
        self.table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(table_device or f"cuda:{device}")
        self.out8 = DeviceBuffer(self.out8_ptr, (2, n_slots, H), 2, "ep_out8")
        assert ctypes.sizeof(table) == 4 * EP_PEERS_WORDS
        self.peers = DeviceBuffer(self.table.data_ptr(), (EP_PEERS_WORDS,), 4, "ep_peers")

    def slots(self, topk):
        """The routed slots this rank computes."""
        return ep_slots(self.rank, self.world, topk)

    def close(self):
        """Release the mappings and the buffers; call after a barrier of all ranks (a peer may
        still be writing into this rank's buffers until then)."""
        for p in self.opened:
            mk.ep_ipc_close(p)
        self.opened = []
        for p in (self.out8_ptr, self.ctr_ptr):
            if p:
                mk.ep_free(p)
        self.out8_ptr = self.ctr_ptr = None
