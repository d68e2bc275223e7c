"""Process-group helpers: one process per GPU, torch.distributed for plumbing.

Launch with ``torchrun --nproc-per-node N --master-addr 127.0.0.1 ...``; every
helper also works unlaunched (world of 1).
"""
import datetime
import os
import uuid

import torch
import torch.distributed as dist


def env_rank():
    return int(os.environ.get("RANK", "0"))


def env_world():
    return int(os.environ.get("WORLD_SIZE", "1"))


def env_local_rank():
    return int(os.environ.get("LOCAL_RANK", "0"))


def init(backend=None, timeout_s=120.0, device=True):
    """Initialises the default process group from torchrun's environment (no-op
    for a world of 1 unless MASTER_ADDR is set).  Returns (rank, world)."""
    world = env_world()
    if device and torch.cuda.is_available():
        torch.cuda.set_device(env_local_rank() % max(torch.cuda.device_count(), 1))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl" and torch.cuda.is_available():
            kwargs["device_id"] = torch.device("cuda", torch.cuda.current_device())
        dist.init_process_group(**kwargs)
    return rank(), world_size()


def rank(group=None):
    return dist.get_rank(group) if dist.is_initialized() else 0


def world_size(group=None):
    return dist.get_world_size(group) if dist.is_initialized() else 1


def barrier(group=None):
    if dist.is_initialized() and world_size(group) > 1:
        if dist.get_backend(group) == "nccl":
            dist.barrier(group=group, device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier(group=group)


def broadcast_object(obj, src=0, group=None):
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
    if not dist.is_initialized() or world_size(group) == 1:
        return [obj]
    out = [None] * world_size(group)
    dist.all_gather_object(out, obj, group=group)
    return out
