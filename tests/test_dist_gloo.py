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


# ------------------------------------------------------------------------------------- LayerGrads
def _fake_fn():
    """A CPU stand-in for the fused MLP's backward contract: each parameter's gradient is written into the
    storage mx_dp.grad_out hands out (the bucket slice), or allocated when there is none."""
    import mx_dp

    class F(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x, scale, *ps):
            ctx.ps, ctx.scale = ps, scale
            return x.clone()

        @staticmethod
        def backward(ctx, dy):
            outs = []
            for k, p in enumerate(ctx.ps):
                v = torch.full(p.shape, float(k + 1)) * ctx.scale * dy.sum()
                g = mx_dp.grad_out(p)
                if g is None:
                    g = v
                else:
                    g.copy_(v)
                outs.append(g)
            return (dy, None, *outs)
    return F


def _layer_params(n_layers=3):
    return [[torch.zeros(3, 4, requires_grad=True), torch.zeros(5, requires_grad=True)] for _ in range(n_layers)]


def test_layer_grads_adopts_slices_without_copy():
    import mx_dp
    F = _fake_fn()
    ps = _layer_params()
    lg = mx_dp.LayerGrads(ps)
    for _ in range(2):          # two steps: the buffer is reused once the gradients are dropped
        x = torch.ones(2, requires_grad=True)
        y = x
        for li, layer in enumerate(ps):
            y = F.apply(y, float(li + 1), *layer)
        lg.begin()
        y.sum().backward()
        lg.finish()
        for li, layer in enumerate(ps):
            for k, p in enumerate(layer):
                assert p.grad.data_ptr() == lg.view(p).data_ptr()
                assert torch.equal(p.grad, torch.full(p.shape, 2.0 * (k + 1) * (li + 1)))
        assert lg.copied == 0 and lg.exchanges == 0   # adopted in place; one process: no collective
        lg.zero()
    lg.close()


def test_layer_grads_copies_in_gradients_made_elsewhere():
    """A parameter whose gradient comes from ordinary torch ops (not through grad_out) is copied into its
    slice when accumulated; a parameter the backward never reaches gets a zero slice."""
    import mx_dp
    a = torch.zeros(4, requires_grad=True)
    b = torch.zeros(2, requires_grad=True)
    unused = torch.zeros(3, requires_grad=True)
    lg = mx_dp.LayerGrads([[a, b, unused]])
    lg.begin()
    ((a * 3.0).sum() + (b * 5.0).sum()).backward()
    lg.finish()
    assert lg.copied == 2
    assert torch.equal(a.grad, torch.full((4,), 3.0)) and torch.equal(b.grad, torch.full((2,), 5.0))
    assert torch.equal(unused.grad, torch.zeros(3))
    assert a.grad.data_ptr() == lg.view(a).data_ptr()
    lg.close()


def _layer_grads_worker(rank, world, port, out, overlap=True):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "train-model-template_b200")]
    import mx_dp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    F = _fake_fn()
    ps = _layer_params(4)
    lg = mx_dp.LayerGrads(ps, overlap=overlap)
    order = []
    orig = lg._accumulated

    def spy(p):
        before = lg.exchanges
        orig(p)
        if lg.exchanges > before:
            order.append(lg.where[id(p)][0])   # the layer whose all-reduce was just issued
    for layer in ps:
        for p in layer:
            p._post_accumulate_grad_hooks.clear()
            p.register_post_accumulate_grad_hook(spy)
    res = []
    for step in range(2):
        x = torch.ones(2, requires_grad=True)
        y = x
        for li, layer in enumerate(ps):
            y = F.apply(y, float(li + 1), *layer)
        lg.begin()
        (y.sum() * (rank + 1 + step)).backward()
        lg.finish()
        res.append({(li, k): p.grad.clone() for li, layer in enumerate(ps) for k, p in enumerate(layer)})
        lg.zero()
    if rank == 0:
        out.put((res, order, lg.exchanges, lg.copied))
    dist.barrier()
    dist.destroy_process_group()


def test_layer_grads_allreduce_per_layer_in_backward_order():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    world = 2
    procs = [ctx.Process(target=_layer_grads_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res, order, exchanges, copied = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert exchanges == 8 and copied == 0
    assert order == [3, 2, 1, 0, 3, 2, 1, 0]          # last layer first: its backward finishes first
    for step, grads in enumerate(res):
        dsum = sum(2.0 * (r + 1 + step) for r in range(world))   # dy.sum() of each rank, summed
        for (li, k), g in grads.items():
            assert torch.allclose(g, torch.full(g.shape, dsum * (k + 1) * (li + 1)))


def test_layer_grads_one_allreduce_after_the_backward():
    """overlap=False: the same sums from one all-reduce of the whole buffer in finish()."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    world = 2
    procs = [ctx.Process(target=_layer_grads_worker, args=(r, world, port, q, False)) for r in range(world)]
    for p in procs:
        p.start()
    res, order, exchanges, copied = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert exchanges == 2 and copied == 0 and order == []     # one per step, none from the hooks
    for step, grads in enumerate(res):
        dsum = sum(2.0 * (r + 1 + step) for r in range(world))
        for (li, k), g in grads.items():
            assert torch.allclose(g, torch.full(g.shape, dsum * (k + 1) * (li + 1)))
