"""Token-sharded data parallelism for the fused MXFP8 MLP: one process per GPU, frozen MX weights
replicated, each rank runs the whole path on its own token shard, and the LoRA A/B gradients are the
only data exchanged (NCCL over NVLink on B200).

The reference is single-GPU and has no distributed code; this module is the host side of the sharding
the fused MLP admits: the MLP is token-wise and row-wise MX quantization is per row, so every shard's
codes, scales and outputs are exactly those of the full batch, and the LoRA gradients (sums over
tokens) of the full batch are the sums of the shards' gradients.

Gradient exchange (``LayerGrads``): the LoRA gradients of all layers live in ONE flat fp32 buffer, a
contiguous slice per layer.  The fused MLP's backward writes each gradient straight into its slice
(``grad_out``), autograd's gradient accumulation adopts that storage as ``p.grad`` without a copy, and
as soon as the last gradient of a layer has been accumulated its slice is summed over the ranks with an
asynchronous all-reduce.  The collective runs on the process group's own stream while the backward of
the next (lower) layer computes; ``finish()`` makes the compute stream wait for all of them.
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


def _distributed(group):
    return dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1


# The LayerGrads whose storage backward passes write into (None: fresh allocations).
_ACTIVE = [None]


def grad_out(p, shape=None):
    """Storage for the gradient of parameter `p` that a backward is about to produce: a fresh view of
    its slice in the active LayerGrads when `p` belongs to it and has no gradient yet (so gradient
    accumulation adopts the view as p.grad), else None (the caller allocates).  `shape` defaults to
    p's shape."""
    lg = _ACTIVE[0]
    if lg is None:
        return None
    return lg.slot(p, shape)


class LayerGrads:
    """Flat fp32 storage of the LoRA gradients of a stack of layers, all-reduced layer by layer.

    layer_params: one list of parameters per layer (fp32, contiguous).  Within a layer, parameters are
    laid out in the given order, so parameters whose gradients one kernel writes as a single block
    (for the fused MLP: A_gate then A_up) sit next to each other.
    """

    def __init__(self, layer_params, device=None, group=None, overlap=True):
        """overlap=True: each layer's slice is all-reduced as soon as its gradients exist, overlapped with the
        backward of the layers below; False: one all-reduce of the whole buffer in finish()."""
        self.group = group
        self.overlap = overlap
        self.layers = [list(ps) for ps in layer_params]
        dev = device if device is not None else self.layers[0][0].device
        self.where = {}                 # id(p) -> (layer index, offset, numel)
        self.spans = []                 # (offset, numel) of each layer's slice
        off = 0
        for li, ps in enumerate(self.layers):
            start = off
            for p in ps:
                self.where[id(p)] = (li, off, p.numel())
                off += p.numel()
            self.spans.append((start, off - start))
        self.flat = torch.zeros(off, dtype=torch.float32, device=dev)
        self.works = []
        self.left = [0] * len(self.layers)
        self.hooks = [p.register_post_accumulate_grad_hook(self._accumulated) for ps in self.layers for p in ps]
        self.exchanges = 0              # all-reduces issued (counts for tests)
        self.copied = 0                 # gradients copied in (not produced in place)

    def view(self, p):
        li, off, n = self.where[id(p)]
        return self.flat[off:off + n].view(p.shape)

    def slot(self, p, shape=None):
        w = self.where.get(id(p))
        if w is None or p.grad is not None or p.dtype != torch.float32:
            return None
        _, off, n = w
        return self.flat[off:off + n].view(shape if shape is not None else p.shape)

    def slot_pair(self, p0, p1, shape):
        """One view covering the slices of p0 and p1 when they are adjacent (p1 right after p0) and both
        take their gradient from this buffer; else None."""
        a, b = self.where.get(id(p0)), self.where.get(id(p1))
        if (a is None or b is None or p0.grad is not None or p1.grad is not None or p0.dtype != torch.float32
                or p1.dtype != torch.float32 or a[1] + a[2] != b[1]):
            return None
        return self.flat[a[1]:a[1] + a[2] + b[2]].view(shape)

    # ------------------------------------------------------------------------------------------ step
    def begin(self):
        """Start a backward pass: every parameter must have no gradient (zero_grad(set_to_none=True)).
        Gradients produced into the buffer are adopted without a copy; any other gradient is copied in
        when it is accumulated."""
        self.works = []
        self.left = [len(ps) for ps in self.layers]
        _ACTIVE[0] = self

    def _accumulated(self, p):
        if _ACTIVE[0] is not self:      # a backward outside begin() / finish(): leave p.grad as it is
            return
        li, off, n = self.where[id(p)]
        g = p.grad
        if g is not None and g.data_ptr() != self.flat.data_ptr() + off * 4:
            self.flat[off:off + n].copy_(g.reshape(-1))   # not produced in place (another backward path)
            p.grad = self.flat[off:off + n].view(p.shape)
            self.copied += 1
        self.left[li] -= 1
        if self.left[li] == 0 and self.overlap and _distributed(self.group):
            o, k = self.spans[li]
            self.works.append(dist.all_reduce(self.flat[o:o + k], op=dist.ReduceOp.SUM, group=self.group,
                                              async_op=True))
            self.exchanges += 1

    def finish(self):
        """End of the backward: layers whose parameters got no gradient contribute zeros, then the compute
        stream waits for every layer's all-reduce.  Afterwards p.grad of every parameter is its slice of
        the summed buffer."""
        for li, ps in enumerate(self.layers):
            if self.left[li] == 0:
                continue
            for p in ps:       # a parameter the backward did not reach: zero gradient, same collectives
                if p.grad is None:
                    v = self.view(p)
                    v.zero_()
                    p.grad = v
                    self._accumulated(p)
        _ACTIVE[0] = None
        if not self.overlap and _distributed(self.group):
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
            self.exchanges += 1
        for w in self.works:
            w.wait()
        self.works = []

    def zero(self):
        """Drop the gradients (set to None) so the next backward writes into the buffer again."""
        for ps in self.layers:
            for p in ps:
                p.grad = None

    def close(self):
        for h in self.hooks:
            h.remove()
        self.hooks = []
        if _ACTIVE[0] is self:
            _ACTIVE[0] = None


class GradBucket:
    """One flat fp32 buffer holding the gradients of `params`, all-reduced (sum) in one collective after
    the backward (for callers whose gradients are produced outside the fused MLP)."""

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

    def allreduce(self, group=None):
        """Sum the gradients over the ranks of `group` and write the sums back into p.grad (blocking on
        the host only as far as the collective's launch; the compute stream is ordered after it)."""
        self.pack()
        if _distributed(group):
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
        self.unpack()
