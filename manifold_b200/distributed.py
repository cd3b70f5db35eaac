"""Data parallelism for the recurrence: batch sharding and the gradient
all-reduce of the BPTT configuration.

The reference has no distributed code (no torch.distributed / NCCL call
site).  Rows of the batch are independent through the whole recurrence, so
inference and decode shard by batch with no collective; training adds one
collective, the all-reduce (mean) of the parameter gradients, issued in
buckets so several transfers are in flight at once.  The backend is the
process group's: NCCL over NVLink/NVSwitch on GPUs, gloo on CPU.
"""
import torch
import torch.distributed as dist


def shard_rows(t, rank, world, dim=0):
    """This rank's contiguous slice of a batch-major tensor."""
    n = t.shape[dim]
    per = (n + world - 1) // world
    return t.narrow(dim, min(rank * per, n), max(0, min(per, n - rank * per)))


def allreduce_gradients(params, bucket_bytes=32 << 20, group=None):
    """Average .grad of `params` over the process group in place.

    Gradients are flattened into buckets of about `bucket_bytes`; every
    bucket's all-reduce is started before any is waited on.  Parameters
    without a gradient are skipped (the same on every rank by construction).
    """
    world = dist.get_world_size(group)
    grads = [p.grad for p in params if p.grad is not None]
    if world == 1 or not grads:
        return
    buckets, cur, size = [], [], 0
    for g in grads:
        cur.append(g)
        size += g.numel() * g.element_size()
        if size >= bucket_bytes:
            buckets.append(cur)
            cur, size = [], 0
    if cur:
        buckets.append(cur)
    flats, works = [], []
    for b in buckets:
        flat = torch.cat([g.reshape(-1) for g in b])
        flats.append(flat)
        works.append(dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=True))
    for b, flat, w in zip(buckets, flats, works):
        w.wait()
        flat.div_(world)
        off = 0
        for g in b:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n
