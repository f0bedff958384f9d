"""Token-sharded data parallelism on CPU ranks (gloo, world size 2): the sum all-reduce of the shards'
LoRA gradients equals the full batch's gradients (oracle math), shards tile the batch, and a rank that
fails before the collective makes the other rank's all-reduce fail with an error instead of hanging."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_tile_the_batch():
    import mx_dp
    for T in (1, 77, 128, 1000, 16384, 142336):
        for world in (1, 2, 4, 8):
            spans = [mx_dp.shard_rows(T, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b
            for a, b in spans[:-1]:
                assert a % 128 == 0 and (b - a) % 128 == 0 or b == T


def _case():
    from oracle import mx_oracle as O
    rng = np.random.default_rng(0)
    T, H, N, r = 256, 128, 256, 16
    bf = lambda a: O.bf16_round(a.astype(np.float32))  # noqa: E731
    W = O.MXWeights(bf(rng.standard_normal((N, H)) * 0.02), bf(rng.standard_normal((N, H)) * 0.02),
                    bf(rng.standard_normal((H, N)) * 0.02))
    lora = [(rng.standard_normal(s) * 0.01).astype(np.float32) for s in ((r, H), (N, r), (r, H), (N, r), (r, N), (H, r))]
    x = bf(rng.standard_normal((T, H)))
    dy = bf(rng.standard_normal((T, H)))
    return O, W, lora, x, dy


NAMES = ("dAg", "dBg", "dAu", "dBu", "dAd", "dBd")


def _worker(rank, world, port, out):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "train-model-template_b200")]
    import mx_dp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O, W, lora, x, dy = _case()
    a, b = mx_dp.shard_rows(x.shape[0], world, rank)
    y, ctx = O.mlp_forward(x[a:b], W, *lora, 2.0, 2.0, 2.0)
    g = O.mlp_backward(dy[a:b], ctx)
    params = [torch.zeros(lo.shape, requires_grad=True) for lo in lora]
    for p, k in zip(params, NAMES):
        p.grad = torch.from_numpy(np.ascontiguousarray(g[k], dtype=np.float32))
    mx_dp.GradBucket(params).allreduce()
    if rank == 0:
        out.put({k: p.grad.numpy().copy() for p, k in zip(params, NAMES)})
    dist.barrier()
    dist.destroy_process_group()


def test_allreduce_of_shard_grads_equals_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    O, W, lora, x, dy = _case()
    y, c = O.mlp_forward(x, W, *lora, 2.0, 2.0, 2.0)
    full = O.mlp_backward(dy, c)
    for k in NAMES:
        # per-shard grads are rounded like the reference (bf16 for dA / dB_down) before the sum
        assert O.rel_fro(got[k], full[k]) < 5e-3, k


def _failing_worker(rank, world, port, out):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "train-model-template_b200")]
    import mx_dp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)   # the rank dies between steps, before the gradient exchange
    p = torch.zeros(4, requires_grad=True)
    p.grad = torch.ones(4)
    try:
        mx_dp.GradBucket([p]).allreduce()
        out.put("completed")
    except Exception as e:   # gloo reports the lost peer / timeout as an error
        out.put("error: " + type(e).__name__)


def test_dead_rank_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res.startswith("error"), res
