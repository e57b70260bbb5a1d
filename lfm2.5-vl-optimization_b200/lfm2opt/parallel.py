"""Multi-GPU plumbing for the large-M W8A8 work: one process per GPU, torch.distributed (NCCL over NVLink/NVSwitch).

Two strategies, and no others (the reference is single-GPU; these are the north star's additions):

  row sharding   tokens are independent (per-token scales are row-local), so the rows of a large-M batch are split
                 evenly across ranks and every rank runs the full layer stack on its rows with a replica of the
                 weights. No data-path collective.
  N-split head   the 2048 -> 65536 lm_head is split by output rows: rank r holds weight rows [r V/g, (r+1) V/g),
                 computes its logits slab [M, V/g] and an all-gather assembles [g, M, V/g] on every rank. M is cut
                 into chunks so the all-gather of chunk c (NCCL, on its own stream) overlaps the GEMM of chunk c+1.

The GEMM is injected (`linear`), so the host logic runs unchanged on CPU ranks (gloo) in the tests.
"""

from dataclasses import dataclass

import torch
import torch.distributed as dist


def shard_rows(total: int, world: int, rank: int):
    """(start, count) of rank's contiguous share of `total` rows; the first total % world ranks take one extra."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def split_vocab(V: int, world: int):
    """Per-rank vocabulary slab width for the N-split head (V must divide evenly)."""
    if V % world:
        raise ValueError(f"vocabulary {V} does not split evenly over {world} ranks")
    return V // world


@dataclass
class HeadShard:
    """This rank's slab of the lm_head weight rows."""

    rank: int
    world: int
    V: int
    lo: int
    hi: int


def head_shard(V: int, world: int, rank: int) -> HeadShard:
    w = split_vocab(V, world)
    return HeadShard(rank, world, V, rank * w, (rank + 1) * w)


class NSplitHead:
    """lm_head N-split across the ranks of `group` with a chunked, overlapped all-gather.

    linear(x [m, K]) -> [m, V/g] computes this rank's logits slab (e.g. an Int8Linear over the weight rows
    head_shard(...).lo:hi). __call__(x [M, K]) returns the gathered logits as one flat bf16 buffer laid out
    chunk-major: for chunk c (rows shard_rows(M, chunks, c)) a [g, rows_c, V/g] block, exactly as the all-gather
    of that chunk writes it, so no copy follows the collective. `as_rows(buf, M)` materialises [M, V] (tests and
    consumers that want row-major logits). Each chunk's all-gather is issued asynchronously right after its GEMM;
    NCCL runs it on its own stream while the next chunk's GEMM runs on the current stream. Every rank must call
    with the same M (the collectives are matched in order). on_chunk(off, dst, work), if given, is called as each chunk
    is enqueued: off = its offset in the flat buffer, dst = its [g * rows, V/g] block, work = its all-gather handle
    (None on one rank: dst is then complete in stream order on the current stream), so a consumer can start on a chunk
    (e.g. copy it to the host on another stream after work.wait() there) while later chunks compute. wait=False returns
    before the current stream waits for the gathers (call wait() later), so independent work can be enqueued first.
    """

    def __init__(self, linear, V: int, group=None, chunks: int = 4):
        self.linear = linear
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.V = V
        self.slab = split_vocab(V, self.world)
        self.chunks = max(1, chunks)

    def chunk_bounds(self, M: int):
        return [shard_rows(M, self.chunks, c) for c in range(self.chunks)]

    def __call__(self, x: torch.Tensor, out: torch.Tensor = None, on_chunk=None, wait: bool = True) -> torch.Tensor:
        M = x.shape[0]
        if out is None:
            out = torch.empty(self.world * M * self.slab, device=x.device, dtype=torch.bfloat16)
        works = []
        keep = []  # the chunks' local slabs stay referenced until wait(): see there
        off = 0
        for start, cnt in self.chunk_bounds(M):
            if cnt == 0:
                continue
            local = self.linear(x[start:start + cnt]).contiguous()  # [cnt, slab] on the current stream
            keep.append(local)
            dst = out[off:off + self.world * cnt * self.slab].view(self.world * cnt, self.slab)
            c_off = off
            off += self.world * cnt * self.slab
            if self.world == 1:
                dst.copy_(local)
                if on_chunk is not None:
                    on_chunk(c_off, dst, None)
                continue
            works.append(dist.all_gather_into_tensor(dst, local, group=self.group, async_op=True))
            if on_chunk is not None:
                on_chunk(c_off, dst, works[-1])
        self._works, self._keep = works, keep
        if wait:
            self.wait()
        return out

    def wait(self):
        """Make the current stream wait for the all-gathers of the last call (the call does this itself unless it was
        made with wait=False, which lets the caller enqueue other work first while the gathers proceed). The local
        slabs the gathers read are released only here, after the current stream has waited: an on_chunk consumer that
        waits on another stream would otherwise let the caching allocator hand their memory to new work on the current
        stream while NCCL still reads it."""
        for w in getattr(self, "_works", []):
            w.wait()
        self._works, self._keep = [], []

    def as_rows(self, buf: torch.Tensor, M: int) -> torch.Tensor:
        """Chunk-major gathered buffer -> [M, V] (a copy)."""
        rows = []
        off = 0
        for start, cnt in self.chunk_bounds(M):
            if cnt == 0:
                continue
            blk = buf[off:off + self.world * cnt * self.slab].view(self.world, cnt, self.slab)
            off += self.world * cnt * self.slab
            rows.append(blk.permute(1, 0, 2).reshape(cnt, self.world * self.slab))
        return torch.cat(rows, 0)
