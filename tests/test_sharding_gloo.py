"""Host-side sharding logic on 2 CPU ranks (gloo): column-sharded weight-only
projections and KV-head-sharded attention reassemble exactly the single-rank
result.  The per-rank compute is the CPU oracle standing in for the CUDA kernel
(these tests need no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _linear_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from conftest import load_package
    import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        load_package()
        from onnx_light_b200 import sharding
        K, N, M, bs = 128, 96, 3, 32
        codes = O.randint(1, (K * N,), -8, 7).reshape(K, N)
        scale = O.rand_uniform(2, (K // bs, N), 0.01, 0.02)
        a = O.randn(3, (M, K))

        def compute(a_t, w_codes, s, zp):
            wq = O.dequantize_linear(O.pack_bits(w_codes.numpy(), 4), O.INT4, w_codes.shape,
                                     s.numpy(), O.FLOAT, s.shape, None, None, 0)
            return torch.from_numpy(O.matmul(a_t.numpy(), wq, O.FLOAT))

        b, e = sharding.shard_range(N, world, rank)
        lin = sharding.ShardedLinear(torch.from_numpy(codes[:, b:e].copy()),
                                     torch.from_numpy(scale[:, b:e].copy()), None, N, world, compute)
        y = lin(torch.from_numpy(a)).numpy()
        full = O.matmul(a, O.dequantize_linear(O.pack_bits(codes, 4), O.INT4, (K, N), scale, O.FLOAT,
                                               (K // bs, N), None, None, 0), O.FLOAT)
        q.put((rank, bool(np.array_equal(y, full))))
    finally:
        dist.destroy_process_group()


def _attention_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from conftest import load_package
    import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        load_package()
        from onnx_light_b200 import sharding
        B, Hq, Hkv, L, D = 2, 8, 4, 17, 16
        qf = O.randn(5, (B, Hq, 1, D), 0, 0.5)
        kf = O.randn(6, (B, Hkv, L, D), 0, 0.5)
        vf = O.randn(7, (B, Hkv, L, D), 0, 0.5)
        kb, ke, qb, qe = sharding.kv_head_range(Hkv, Hq, world, rank)
        local = O.attention_f32(qf[:, qb:qe], kf[:, kb:ke], vf[:, kb:ke], is_causal=True, past_len=L - 1)
        y = sharding.gather_heads(torch.from_numpy(local), world).numpy()
        full = O.attention_f32(qf, kf, vf, is_causal=True, past_len=L - 1)
        q.put((rank, bool(np.array_equal(y, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("worker", [_linear_worker, _attention_worker])
def test_two_rank_sharding_reassembles_single_rank_result(worker):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(results.values()), results


def test_shard_range_rules(b2):
    from onnx_light_b200 import sharding
    assert sharding.shard_range(11008, 8, 7) == (9632, 11008)
    assert sharding.kv_head_range(8, 32, 4, 1) == (2, 4, 8, 16)
    with pytest.raises(ValueError):
        sharding.shard_range(10, 3, 0)
