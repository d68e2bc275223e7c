"""Process-group helpers: one process per GPU, torch.distributed for plumbing.

Launch with ``torchrun --nproc-per-node N --master-addr 127.0.0.1 ...``; every
helper also works unlaunched (world of 1).
"""
import datetime
import os
import uuid

import torch
import torch.distributed as dist


# Launcher variables, first match wins.  torchrun's come first: under torchrun
# inside a SLURM allocation every child shares SLURM_LOCALID but has its own
# LOCAL_RANK.  The MPI and SLURM names are the ones the reference's launch
# discovery reads (apps/README.md:297-300 of AMDResearch/kiwi).
RANK_VARS = ("RANK", "OMPI_COMM_WORLD_RANK", "PMI_RANK", "SLURM_PROCID")
WORLD_VARS = ("WORLD_SIZE", "OMPI_COMM_WORLD_SIZE", "PMI_SIZE", "SLURM_NTASKS")
LOCAL_RANK_VARS = ("LOCAL_RANK", "OMPI_COMM_WORLD_LOCAL_RANK", "MPI_LOCALRANKID", "SLURM_LOCALID")


def _first_env(names, default, env=None):
    env = os.environ if env is None else env
    for n in names:
        v = env.get(n)
        if v not in (None, ""):
            return int(v)
    return default


def env_rank(env=None):
    """Global rank from the launcher's variables (RANK_VARS), 0 if none is set."""
    return _first_env(RANK_VARS, 0, env)


def env_world(env=None):
    """World size from the launcher's variables (WORLD_VARS), 1 if none is set."""
    return _first_env(WORLD_VARS, 1, env)


def env_local_rank(env=None):
    """Rank within the node (LOCAL_RANK_VARS), 0 if none is set."""
    return _first_env(LOCAL_RANK_VARS, 0, env)


def init(backend=None, timeout_s=120.0, device=True):
    """Initialises the default process group from the launcher's environment
    (torchrun, or mpirun / srun through RANK_VARS, WORLD_VARS and
    LOCAL_RANK_VARS; MASTER_ADDR defaults to 127.0.0.1 and MASTER_PORT to 29500
    when the launcher sets neither).  No-op for a world of 1.  Returns (rank, world)."""
    world = env_world()
    if device and torch.cuda.is_available():
        torch.cuda.set_device(env_local_rank() % max(torch.cuda.device_count(), 1))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s),
                      rank=env_rank(), world_size=world)
        if backend == "nccl" and torch.cuda.is_available():
            kwargs["device_id"] = torch.device("cuda", torch.cuda.current_device())
        dist.init_process_group(**kwargs)
    return rank(), world_size()


def rank(group=None):
    """This process's rank in `group` (0 without a process group)."""
    return dist.get_rank(group) if dist.is_initialized() else 0


def world_size(group=None):
    """Size of `group` (1 without a process group)."""
    return dist.get_world_size(group) if dist.is_initialized() else 1


def barrier(group=None):
    """Host barrier over `group` (a no-op for a world of 1)."""
    if dist.is_initialized() and world_size(group) > 1:
        if dist.get_backend(group) == "nccl":
            dist.barrier(group=group, device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier(group=group)


def broadcast_object(obj, src=0, group=None):
    """`obj` from rank `src` of `group` on every rank."""
    if not dist.is_initialized() or world_size(group) == 1:
        return obj
    lst = [obj]
    dist.broadcast_object_list(lst, src=dist.get_global_rank(group, src) if group is not None else src, group=group)
    return lst[0]


def job_id(group=None):
    """A token unique to this group instance (names the FD-exchange sockets)."""
    return broadcast_object(uuid.uuid4().hex[:16] if rank(group) == 0 else None, 0, group)


def max_over_ranks(value, group=None):
    """Max of a float over ranks (device timing is reported as the max)."""
    if not dist.is_initialized() or world_size(group) == 1:
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def all_gather_objects(obj, group=None):
    """Every rank's `obj`, in rank order."""
    if not dist.is_initialized() or world_size(group) == 1:
        return [obj]
    out = [None] * world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out
