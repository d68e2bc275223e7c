"""Process-group bootstrap and host-side failure detection on CPU (gloo ranks).

Covers launcher discovery (torchrun, mpirun and srun variable names), the
helpers every benchmark uses for cross-rank timing, and the failure modes the
reference leaves as hangs: a peer that never joins (bootstrap ends with a
timeout error) and a peer that exits between steps (the next collective ends
with an error instead of waiting forever).
"""
import multiprocessing as mp
import os
import socket
import time

import pytest

from kiwi_b200.utils import dist as kdist


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_launcher_variable_precedence():
    assert kdist.env_local_rank({"SLURM_LOCALID": "3"}) == 3
    assert kdist.env_local_rank({"SLURM_LOCALID": "0", "LOCAL_RANK": "2"}) == 2
    assert kdist.env_local_rank({"OMPI_COMM_WORLD_LOCAL_RANK": "5", "MPI_LOCALRANKID": "1"}) == 5
    assert kdist.env_local_rank({}) == 0
    assert kdist.env_rank({"OMPI_COMM_WORLD_RANK": "7"}) == 7
    assert kdist.env_rank({"PMI_RANK": "4", "SLURM_PROCID": "9"}) == 4
    assert kdist.env_world({"SLURM_NTASKS": "16"}) == 16
    assert kdist.env_world({"WORLD_SIZE": "2", "OMPI_COMM_WORLD_SIZE": "8"}) == 2
    assert kdist.env_world({"WORLD_SIZE": ""}) == 1


def _clean_env():
    for n in kdist.RANK_VARS + kdist.WORLD_VARS + kdist.LOCAL_RANK_VARS + ("MASTER_ADDR", "MASTER_PORT"):
        os.environ.pop(n, None)


def _member(env, q, mode):
    _clean_env()
    os.environ.update(env)
    try:
        rank, world = kdist.init(backend="gloo", timeout_s=4.0, device=False)
        if mode == "ok":
            kdist.barrier()
            got = kdist.all_gather_objects((rank, kdist.env_local_rank()))
            mx = kdist.max_over_ranks(float(rank) + 0.5)
            jid = kdist.job_id()
            q.put(("ok", rank, world, got, mx, jid))
        elif mode == "leave":
            kdist.barrier()
            if rank == 1:
                q.put(("left", rank))
                q.close()
                q.join_thread()  # flush before leaving
                os._exit(0)  # leaves between steps, nothing in flight
            time.sleep(0.5)
            t0 = time.monotonic()
            try:
                kdist.barrier()
                q.put(("no-error", rank, time.monotonic() - t0))
            except Exception as e:  # noqa: BLE001 - any error type is a detection
                q.put(("error", rank, time.monotonic() - t0, type(e).__name__))
        if kdist.dist.is_initialized():
            kdist.dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put(("init-error", type(e).__name__, str(e)[:200]))


def _run(envs, mode, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_member, args=(env, q, mode)) for env in envs]
    for p in ps:
        p.start()
    out = []
    deadline = time.monotonic() + timeout
    while len(out) < len(ps) and time.monotonic() < deadline:
        try:
            out.append(q.get(timeout=1.0))
        except Exception:  # noqa: BLE001 - queue.Empty
            if not any(p.is_alive() for p in ps) and q.empty():
                break
    for p in ps:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
            p.join()
    return out


@pytest.mark.parametrize("launcher", ["mpirun", "srun"])
def test_two_gloo_ranks_from_launcher_variables(launcher):
    port = str(_free_port())
    if launcher == "mpirun":
        envs = [{"OMPI_COMM_WORLD_RANK": str(r), "OMPI_COMM_WORLD_SIZE": "2",
                 "OMPI_COMM_WORLD_LOCAL_RANK": str(r), "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": port}
                for r in range(2)]
    else:
        envs = [{"SLURM_PROCID": str(r), "SLURM_NTASKS": "2", "SLURM_LOCALID": str(r),
                 "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": port} for r in range(2)]
    out = _run(envs, "ok")
    assert len(out) == 2, out
    assert all(o[0] == "ok" for o in out), out
    by_rank = {o[1]: o for o in out}
    assert set(by_rank) == {0, 1}
    for r, o in by_rank.items():
        assert o[2] == 2
        assert o[3] == [(0, 0), (1, 1)]
        assert o[4] == 1.5
    assert by_rank[0][5] == by_rank[1][5]  # one job id for the whole group


def test_peer_that_never_joins_ends_bootstrap_with_an_error():
    port = str(_free_port())
    env = {"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0", "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": port}
    t0 = time.monotonic()
    out = _run([env], "ok", timeout=40)
    assert out and out[0][0] == "init-error", out
    assert time.monotonic() - t0 < 40


def test_peer_that_leaves_between_steps_is_detected_by_the_next_collective():
    port = str(_free_port())
    envs = [{"RANK": str(r), "WORLD_SIZE": "2", "LOCAL_RANK": str(r), "MASTER_ADDR": "127.0.0.1",
             "MASTER_PORT": port} for r in range(2)]
    out = _run(envs, "leave", timeout=60)
    kinds = sorted(o[0] for o in out)
    assert kinds == ["error", "left"], out
    err = next(o for o in out if o[0] == "error")
    assert err[1] == 0 and err[2] < 30.0
