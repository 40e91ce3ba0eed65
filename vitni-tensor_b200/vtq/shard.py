"""Output-row sharding of a linear across the ranks of one node.

Every output row of the reference's linears is an independent reduction
(src/ops/quant.rs:1373-1377), so a rank that owns rows [a, b) computes
exactly the reference's y[a:b]. Shards are contiguous, balanced row ranges;
the full y is reassembled by an all-gather of the per-rank shards (NCCL over
NVLink on GPUs, gloo on CPU in the tests).
"""
from __future__ import annotations


def row_range(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced shard [a, b) of `rows` for `rank` of `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    return rank * rows // world, (rank + 1) * rows // world


def shard_rows(rows: int, world: int) -> list[tuple[int, int]]:
    return [row_range(rows, world, r) for r in range(world)]


def gather_rows(local, rows: int, batch: int, group=None):
    """All-gather per-rank y shards ([batch][b - a] each) into y [batch][rows].

    `local` is a torch tensor on this rank's device (cuda for NCCL, cpu for
    gloo). Shards are padded to the largest shard so the collective moves
    equal-sized buffers; padding is dropped on reassembly.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    ranges = shard_rows(rows, world)
    width = max(b - a for a, b in ranges)
    buf = torch.zeros(batch, width, dtype=local.dtype, device=local.device)
    mine = ranges[dist.get_rank(group)]
    buf[:, : mine[1] - mine[0]] = local.reshape(batch, mine[1] - mine[0])
    out = torch.empty(world * batch, width, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, buf.contiguous(), group=group)
    out = out.view(world, batch, width)
    parts = [out[r, :, : b - a] for r, (a, b) in enumerate(ranges)]
    return torch.cat(parts, dim=1).contiguous()


class ShardedLinear:
    """Rows [a, b) of one weight resident on this rank's device; __call__
    computes the local rows with the sm_100a kernels and all-gathers y."""

    def __init__(self, ctx, dtype: int, data, in_feat: int, out_feat: int, group=None):
        import torch.distributed as dist
        self.ctx, self.dtype, self.in_feat, self.out_feat, self.group = (
            ctx, dtype, in_feat, out_feat, group)
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.a, self.b = row_range(out_feat, self.world, self.rank)
        self.weight = ctx.upload(dtype, data, in_feat, out_feat, self.a, self.b)

    def __call__(self, x, batch: int = 1):
        """x: cuda float32 tensor [batch][in_feat]; returns y [batch][out_feat] on cuda."""
        import torch
        y_local = torch.empty(batch, self.b - self.a, dtype=torch.float32, device=x.device)
        self.ctx.linear_ptr(self.weight, x.data_ptr(), y_local.data_ptr(), batch)
        return gather_rows(y_local, self.out_feat, batch, self.group)
