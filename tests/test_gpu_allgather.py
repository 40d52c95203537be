"""b2_allgather_cols on two GPUs (one process each, CUDA IPC peer buffers set
up through a gloo process group): the gathered output equals the
concatenation of the slices, in direct calls and CUDA-graph replays, and a
rank that never arrives makes the other's bounded wait run out and report
itself (code 1) instead of hanging.  Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, result):
    import sys
    sys.path.insert(0, HERE)
    import torch.distributed as dist
    from conftest import load_package
    b2 = load_package()  # noqa: F841
    from onnx_light_b200 import _capi
    from onnx_light_b200.sharding import PeerGroup
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    lib = _capi.lib()
    lib.b2_kernel_status(1)
    peers = PeerGroup()
    M, n = 5, 64
    full = peers.buffer("y", (M, n * world), torch.float16)
    local = (torch.arange(M * n, device="cuda", dtype=torch.float32).view(M, n) + 1000 * rank).half()
    want = torch.cat([(torch.arange(M * n, device="cuda", dtype=torch.float32).view(M, n)
                       + 1000 * r).half() for r in range(world)], dim=1)
    ok = True
    if mode == "gather":
        peers.gather("y", local)
        torch.cuda.synchronize()
        ok &= torch.equal(full, want)
        # captured and replayed: the generation advances on the device
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        local2 = local + 1
        with torch.cuda.graph(g, stream=s):
            peers.gather("y", local2)
        for _ in range(3):
            with torch.cuda.stream(s):
                g.replay()
        torch.cuda.synchronize()
        ok &= torch.equal(full, want + 1)
        ok &= lib.b2_kernel_status(1) == 0
        del g
    else:  # rank 1 never issues its gather: rank 0's wait runs out (5 s) and reports
        if rank == 0:
            peers.gather("y", local)
            torch.cuda.synchronize()
            ok &= lib.b2_kernel_status(1) == 1
        dist.barrier()
    peers.close()
    dist.destroy_process_group()
    result[rank] = bool(ok)


@pytest.mark.parametrize("mode", ["gather", "absent_peer_times_out"])
def test_allgather_cols_two_gpus(cuda, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    result = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(result) == {0: True, 1: True}
