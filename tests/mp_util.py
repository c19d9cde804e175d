"""Spawn helper for multi-process CPU tests (gloo ranks on 127.0.0.1)."""

import os
import socket
import traceback

import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(fn, rank, world, port, q, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        q.put((rank, fn(rank, world, *args)))
    except BaseException:
        q.put((rank, RuntimeError(traceback.format_exc())))


def run_ranks(fn, world: int, *args, timeout: float = 300.0) -> dict:
    """Run ``fn(rank, world, *args)`` in ``world`` spawned processes; returns {rank: result} and
    re-raises the first rank's exception."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q, args)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=timeout)
            out[r] = v
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for r in sorted(out):
        if isinstance(out[r], BaseException):
            raise out[r]
    return out
