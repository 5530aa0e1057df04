"""Expert parallelism over the ranks of one node (one process per GPU), by slot.

Every rank runs the whole decode graph: attention, the dense layer 0, the embedding, the head and
the router are replicated (the router is deterministic, so all ranks route alike). Every rank
holds every expert's weights (31 GB in all, far below one GPU's 180 GB), so the eight slots of a
token (the six routed experts, then the two shared ones) are dealt round-robin: rank r of N
computes the slots s with s mod N = r, whatever experts the router picked. The ranks then stay
within one slot of each other at batch 1, where sharding by expert id leaves a rank idle whenever
the top-6 experts cluster on another.

Each down-projection task sends the rows of its rank's slots to every peer as tagged 64-bit words
(two BF16 rows per word, the iteration's tag in the high half; one store each), reads the other
slots' rows from its own words as their tags arrive, and adds the eight slots in slot order: the
result is the one-GPU result bit for bit. The words are plain device memory from the library
(cudaMalloc), mapped into the peers with CUDA IPC; no multicast object is involved. Handles travel
over the process group."""
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


def exchange_bytes(n_slots, H, n_layers):
    """One rank's exchange words: [2][n_layers][n_slots][H / 2] of 8 bytes (3.4 MB at REAL_DIMS)."""
    return 2 * n_layers * n_slots * (H // 2) * 8


class EpGroup:
    """This rank's exchange words, its peers' (opened through IPC) and the device peer table.

    n_slots, H: the slot rows exchanged; n_layers: MoE layers (one set of words each).
    all_gather(obj) -> list of every rank's obj (torch.distributed.all_gather_object on the node's
    group). Every rank must then launch the same iteration counts (the words' tags count them)."""

    def __init__(self, rank, world, device, n_slots, H, n_layers, all_gather, table_device=None):
        import torch

        assert 1 <= world <= mk.EP_MAX_RANKS and H % 2 == 0
        self.rank, self.world, self.device = rank, world, device
        self.n_slots, self.H, self.n_layers = n_slots, H, n_layers
        self.xch_bytes = exchange_bytes(n_slots, H, max(1, n_layers))
        self.xch_ptr = mk.ep_alloc(device, self.xch_bytes)
        handles = all_gather(mk.ep_ipc_handle(self.xch_ptr))
        self.peer_xch, self.opened = [], []
        for r, hd in enumerate(handles):
            if r == rank:
                self.peer_xch.append(self.xch_ptr)
            else:
                p = mk.ep_ipc_open(device, hd)
                self.opened.append(p)
                self.peer_xch.append(p)
        table = mk.MkEpPeers()
        for r in range(world):
            table.xch[r] = self.peer_xch[r]
        table.nranks, table.rank = world, rank
        table.n_layers, table.n_slots, table.hidden = max(1, n_layers), n_slots, H
        raw = bytes(ctypes.string_at(ctypes.addressof(table), ctypes.sizeof(table)))
        self.table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(table_device or f"cuda:{device}")
        assert ctypes.sizeof(table) == 4 * EP_PEERS_WORDS
        self.peers = DeviceBuffer(self.table.data_ptr(), (EP_PEERS_WORDS,), 4, "ep_peers")

    def slots(self):
        """The slots this rank computes (routed and shared)."""
        return ep_slots(self.rank, self.world, self.n_slots)

    def close(self):
        """Release the mappings and the words; call after a barrier of all ranks (a peer may still
        be writing into this rank's words until then)."""
        for p in self.opened:
            mk.ep_ipc_close(p)
        self.opened = []
        if self.xch_ptr:
            mk.ep_free(self.xch_ptr)
        self.xch_ptr = None
