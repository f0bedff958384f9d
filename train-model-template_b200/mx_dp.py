"""Token-sharded data parallelism for the fused MXFP8 MLP: one process per GPU, frozen MX weights
replicated, each rank runs the whole path on its own token shard, and the LoRA A/B gradients are the
only data exchanged (one bucketed sum all-reduce per step, NCCL over NVLink on B200).

The reference is single-GPU and has no distributed code; this module is the host side of the sharding
the fused MLP admits: the MLP is token-wise and row-wise MX quantization is per row, so every shard's
codes, scales and outputs are exactly those of the full batch, and the LoRA gradients (sums over
tokens) of the full batch are the sums of the shards' gradients.
"""
import torch
import torch.distributed as dist


def shard_rows(T, world, rank, align=128):
    """Contiguous token range [start, end) of `rank` out of `world`: shards are multiples of `align`
    rows (the MX scale-block height) except the last, and differ by at most `align` rows."""
    blocks = -(-T // align)
    per, extra = divmod(blocks, world)
    b0 = rank * per + min(rank, extra)
    b1 = b0 + per + (1 if rank < extra else 0)
    return min(b0 * align, T), min(b1 * align, T)


class GradBucket:
    """One flat fp32 buffer holding the gradients of `params`, all-reduced (sum) in one collective."""

    def __init__(self, params, device=None):
        self.params = list(params)
        n = sum(p.numel() for p in self.params)
        dev = device if device is not None else self.params[0].device
        self.flat = torch.zeros(n, dtype=torch.float32, device=dev)

    def pack(self):
        off = 0
        for p in self.params:
            k = p.numel()
            if p.grad is None:
                self.flat[off:off + k].zero_()
            else:
                self.flat[off:off + k].copy_(p.grad.reshape(-1))
            off += k
        return self.flat

    def unpack(self):
        off = 0
        for p in self.params:
            k = p.numel()
            g = self.flat[off:off + k].view_as(p)
            if p.grad is None:
                p.grad = g.to(p.dtype).clone()
            else:
                p.grad.copy_(g)
            off += k

    def allreduce(self, group=None, async_op=False):
        """Sum the gradients over the ranks of `group` and write the sums back into p.grad."""
        self.pack()
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            work = dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
            if async_op:
                return work
        self.unpack()
        return None
