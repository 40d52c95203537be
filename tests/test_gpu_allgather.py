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
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
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
    elif mode == "fused_matmul":
        # b2_dequantize_matmul_peer: each rank's int4 decode GEMV stores its
        # column slice into both ranks' outputs; a chain of two sharded
        # calls (the second reads the first's gathered output, waiting for
        # the other rank's slice) matches the oracle's chain on the full
        # weights within the fp16 contract.
        import numpy as np
        import oracle as O
        from util import random_q, scale_raw, to_dev, rel_l2
        K, N = 1024, 512
        nl = N // world
        w1 = random_q(71, (K, N), O.INT4)
        s1 = scale_raw(O.rand_uniform(72, ((K // 128) * N,), 0.002, 0.02), O.FLOAT16).reshape(K // 128, N)
        w2 = random_q(73, (N, K), O.INT4)
        s2 = scale_raw(O.rand_uniform(74, ((N // 128) * K,), 0.002, 0.02), O.FLOAT16).reshape(N // 128, K)
        x = O.f32_to_f16_bits(O.randn(75, (1, K)))
        y1 = O.matmul(x, O.dequantize_linear(w1, O.INT4, (K, N), s1.ravel(), O.FLOAT16, (K // 128, N),
                                              None, None, 0), O.FLOAT16)
        y2 = O.matmul(y1, O.dequantize_linear(w2, O.INT4, (N, K), s2.ravel(), O.FLOAT16, (N // 128, K),
                                              None, None, 0), O.FLOAT16)
        # slice the packed int4 weight by columns on the host (two codes per byte)
        def slice_int4(wq, kk, nn):
            b = np.asarray(wq, np.uint8).reshape(kk, nn // 2)
            return np.ascontiguousarray(b[:, rank * (nn // world) // 2:(rank + 1) * (nn // world) // 2])
        tw1 = b2.QTensor(to_dev(slice_int4(w1, K, N)), O.INT4, (K, nl))
        ts1 = to_dev(np.ascontiguousarray(s1.reshape(-1, N)[:, rank * nl:(rank + 1) * nl]), torch.float16)
        tw2 = b2.QTensor(to_dev(slice_int4(w2, N, K)), O.INT4, (N, K // world))
        ts2 = to_dev(np.ascontiguousarray(s2.reshape(-1, K)[:, rank * (K // world):(rank + 1) * (K // world)]),
                     torch.float16)
        full1 = peers.buffer("y1", (1, N), torch.float16)
        full2 = peers.buffer("y2", (1, K), torch.float16)
        tx = to_dev(x).view(torch.float16).reshape(1, K)
        for _ in range(2):  # twice: the generations advance
            peers.matmul("y1", tx, tw1, ts1)
            peers.matmul("y2", full1, tw2, ts2)
            peers.wait()
            torch.cuda.synchronize()
            got1 = full1.float().cpu().numpy()
            got2 = full2.float().cpu().numpy()
            ok &= rel_l2(got1, O.f16_bits_to_f32(y1)) <= 1e-3
            ok &= rel_l2(got2, O.f16_bits_to_f32(y2)) <= 1e-3
        ok &= lib.b2_kernel_status(1) == 0
    elif mode == "fused_group":
        # b2_dequantize_matmul_group_peer: two projections of the same input in
        # one launch, each stored into both ranks' outputs, then a sharded call
        # on the first one's output; three steps back to back with no wait of
        # their own (the chain orders every overwrite), checked after a wait.
        import numpy as np
        import oracle as O
        from util import random_q, scale_raw, to_dev, rel_l2
        K, N = 1024, 768

        def sliced(seed, kk, nn):
            wq = random_q(seed, (kk, nn), O.INT4)
            sc = scale_raw(O.rand_uniform(seed + 1, ((kk // 128) * nn,), 0.002, 0.02),
                           O.FLOAT16).reshape(kk // 128, nn)
            nl = nn // world
            b = np.asarray(wq, np.uint8).reshape(kk, nn // 2)
            wl = np.ascontiguousarray(b[:, rank * nl // 2:(rank + 1) * nl // 2])
            sl = np.ascontiguousarray(sc[:, rank * nl:(rank + 1) * nl])
            deq = O.dequantize_linear(wq, O.INT4, (kk, nn), sc.ravel(), O.FLOAT16, (kk // 128, nn),
                                      None, None, 0)
            return (b2.QTensor(to_dev(wl), O.INT4, (kk, nl)), to_dev(sl, torch.float16), deq)

        wa, wb, w2 = sliced(81, K, N), sliced(83, K, N), sliced(85, N, K)
        fa = peers.buffer("ya", (2, N), torch.float16)
        fb = peers.buffer("yb", (2, N), torch.float16)
        f2 = peers.buffer("y2", (2, K), torch.float16)
        for step in range(3):
            x = O.f32_to_f16_bits(O.randn(90 + step, (2, K)))
            tx = to_dev(x).view(torch.float16).reshape(2, K)
            peers.matmul_group(["ya", "yb"], tx, [wa[0], wb[0]], [wa[1], wb[1]])
            peers.matmul("y2", fa, w2[0], w2[1])
        peers.wait()
        torch.cuda.synchronize()
        ya = O.matmul(x, wa[2], O.FLOAT16)
        yb = O.matmul(x, wb[2], O.FLOAT16)
        y2 = O.matmul(ya, w2[2], O.FLOAT16)
        for got, want in ((fa, ya), (fb, yb), (f2, y2)):
            ok &= rel_l2(got.float().cpu().numpy(), O.f16_bits_to_f32(want)) <= 1e-3
        ok &= lib.b2_kernel_status(1) == 0
    else:  # rank 1 never issues its gather: rank 0's wait runs out (5 s) and reports
        if rank == 0:
            peers.gather("y", local)
            torch.cuda.synchronize()
            ok &= lib.b2_kernel_status(1) == 1
        dist.barrier()
    peers.close()
    dist.destroy_process_group()
    result[rank] = bool(ok)


@pytest.mark.parametrize("mode", ["gather", "fused_matmul", "fused_group", "absent_peer_times_out"])
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
