"""Host side of tensor parallelism, no GPU: the handle exchange over a real torch.distributed group
(gloo, 2 ranks on 127.0.0.1), its checks, and the C entry points' argument errors."""

import ctypes
import os

import pytest
import torch.multiprocessing as mp

from ggml_compiler_b200.runtime import joined_handles, torch_all_gather


def _rank(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        mine = bytes([rank + 1]) * 64
        q.put((rank, joined_handles(mine, rank, world, torch_all_gather())))
    finally:
        dist.destroy_process_group()


def test_handles_gathered_in_rank_order():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = bytes([1]) * 64 + bytes([2]) * 64
    assert got == {0: want, 1: want}


def test_handle_checks():
    a, b = b"\x01" * 64, b"\x02" * 64
    assert joined_handles(b, 1, 2, lambda x: [a, x]) == a + b
    with pytest.raises(ValueError, match="must return 2 handles"):
        joined_handles(a, 0, 2, lambda x: [x])
    with pytest.raises(ValueError, match="in rank order"):
        joined_handles(a, 0, 2, lambda x: [b, x])
    with pytest.raises(ValueError, match="in rank order"):
        joined_handles(a, 0, 2, lambda x: [x, b"\x02" * 32])


def test_entry_points_reject_bad_arguments(rtlib):
    h = ctypes.create_string_buffer(256)
    assert rtlib.ggml_compiler_b200_tp_init(None, 0, 2, 0, h, len(h)) == -1
    assert "must not be NULL" in rtlib.ggml_compiler_last_error().decode()
    assert rtlib.ggml_compiler_b200_tp_connect(None, h, 128) == -1
    assert "must not be NULL" in rtlib.ggml_compiler_last_error().decode()
