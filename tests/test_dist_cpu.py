"""Multi-process host logic on CPU ranks (gloo, world_size 2): row sharding, the N-split lm_head with its chunked
all-gather, and failure detection on the host (a rank that never joins makes the other rank's collective fail with an
error instead of hanging). The GEMM is the CPU oracle, injected where the GPU run uses Int8Linear."""

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lfm2opt.parallel import NSplitHead, head_shard, shard_rows, split_vocab


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_rows_cover_exactly():
    for total in (0, 1, 7, 65536, 65537):
        for world in (1, 2, 4, 8):
            spans = [shard_rows(total, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == total
            assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)
    with pytest.raises(ValueError):
        split_vocab(65536, 3)
    hs = head_shard(65536, 8, 3)
    assert (hs.lo, hs.hi) == (24576, 32768)


def _oracle_linear(wq, sw):
    import oracle

    def lin(x, out=None):
        xq, sx = oracle.quant_rows_ref(x)
        return oracle.gemm_i8_ref(xq, sx, wq, sw)
    return lin


def _head_worker(rank, world, port, M, V, K, chunks, wait, q):
    os.environ["OMP_NUM_THREADS"] = "1"
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        import oracle
        g = torch.Generator().manual_seed(7)
        w = (torch.randn(V, K, generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        wq, sw = oracle.quantize_int8_ref(w)
        hs = head_shard(V, world, rank)
        head = NSplitHead(_oracle_linear(wq[hs.lo:hs.hi].contiguous(), sw[hs.lo:hs.hi].contiguous()), V, chunks=chunks)
        seen = []

        def on_chunk(off, dst, work):  # a consumer of finished chunks: copies each one as soon as it is gathered
            if work is not None:
                work.wait()
            seen.append((off, dst.reshape(-1).clone()))

        buf = head(x, on_chunk=on_chunk, wait=wait)
        if not wait:  # the gathered slabs' sources stay referenced until wait() and are released there
            assert len(head._keep) == sum(1 for _, c in head.chunk_bounds(M) if c)
            head.wait()
            assert head._keep == [] and head._works == []
        full = head.as_rows(buf, M)
        # the chunks reported tile the buffer in order and hold the final gathered values
        offs = [o for o, _ in seen]
        assert offs == sorted(offs) and offs[0] == 0
        assert sum(v.numel() for _, v in seen) == buf.numel()
        assert all(torch.equal(v, buf[o:o + v.numel()]) for o, v in seen)
        xq, sx = oracle.quant_rows_ref(x)
        ref = oracle.gemm_i8_ref(xq, sx, wq, sw)
        q.put((rank, bool(torch.equal(full, ref)), tuple(full.shape)))
    except Exception as e:  # reported to the parent
        q.put((rank, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,chunks,wait", [(37, 3, True), (64, 4, False), (5, 8, True)])
def test_nsplit_head_gathers_the_full_logits(M, chunks, wait):
    world, V, K = 2, 96, 128
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, world, port, M, V, K, chunks, wait, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in res:
        assert ok, (rank, info)
        assert info == (M, V)


def _absent_peer_worker(rank, world, port, q):
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight, and never joins the next one
    try:
        head = NSplitHead(lambda x, out=None: torch.zeros(x.shape[0], 8, dtype=torch.bfloat16), 16, chunks=2)
        head(torch.zeros(4, 8, dtype=torch.bfloat16))
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, type(e).__name__))


def test_absent_rank_surfaces_as_an_error():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and outcome != "no error", outcome
