"""Data-parallel training over several GPUs of one node (one process per GPU).

LightGBM's data-parallel tree learner (tree_learner=data): every rank holds a contiguous
shard of the rows; after each histogram build the ranks sum the integer child histogram
and its left-row count inside the library -- over peer memory (CUDA IPC mappings of
every rank's accumulators, plain loads, bounded waits) when all ranks can map each
other, else with one NCCL all-reduce per split -- so all ranks grow identical trees.
With wide data (at least 128 features per rank) each rank decodes and scans only its slice
of the features, and the slices' best splits are exchanged before every rank takes the
same pick. The gradient step's scale maxima and root sums are NCCL reductions. The
reference maps tree_learner=data back to serial (crates/lgbm-core/src/config/set.rs:
592-600); this module has no counterpart there.

The NCCL id is made on rank 0 and handed to the other ranks out of band; with
torch.distributed already initialised (any backend, e.g. gloo), `from_torch` does that.
"""

import ctypes

from . import _lib as C

__all__ = ["shard_range", "unique_id", "Communicator", "from_torch"]


def shard_range(num_data, world_size, rank):
    """Rows [begin, end) of `rank`: contiguous shards in rank order, sizes differing by at
    most one. The shards in rank order are the job's global row order."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} of {world_size}")
    return num_data * rank // world_size, num_data * (rank + 1) // world_size


def _nccl_first():
    """Load the NCCL that PyTorch links, if PyTorch is installed, before the library
    looks for one: the library then uses that same NCCL instead of loading a second
    build under the same soname (which would break a later `import torch`)."""
    try:
        import torch  # noqa: F401
    except ImportError:
        pass


def unique_id():
    """A fresh NCCL id (LGBM_B200_COMM_ID_BYTES bytes), made on one rank."""
    _nccl_first()
    buf = (ctypes.c_uint8 * 128)()
    C.check(C.lib().lgbm_b200_comm_unique_id(buf))
    return bytes(buf)


class Communicator:
    """One rank's NCCL communicator on `device` (the library's lgbm_b200_comm)."""

    def __init__(self, device, world_size, rank, uid):
        if len(uid) != 128:
            raise ValueError("NCCL id must be 128 bytes")
        _nccl_first()
        self.device, self.world_size, self.rank = int(device), int(world_size), int(rank)
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        h = ctypes.c_void_p()
        C.check(C.lib().lgbm_b200_comm_create(self.device, self.world_size, self.rank, buf,
                                              ctypes.byref(h)))
        self._handle = h

    def close(self):
        if getattr(self, "_handle", None):
            C.lib().lgbm_b200_comm_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def broadcast_bytes(data, src=0):
    """Send `data` (bytes, significant on `src`) to every rank of the initialised
    torch.distributed group; returns the bytes on every rank."""
    import torch.distributed as dist

    obj = [data if dist.get_rank() == src else None]
    dist.broadcast_object_list(obj, src=src)
    return obj[0]


def from_torch(device):
    """Communicator for this process, with rank and world size taken from the initialised
    torch.distributed group (which carries the NCCL id from rank 0)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(), dist.get_world_size()
    uid = broadcast_bytes(unique_id() if rank == 0 else None, src=0)
    return Communicator(device, world, rank, uid)
