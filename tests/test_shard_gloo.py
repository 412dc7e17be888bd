"""Multi-rank host logic on CPU (gloo, world size 2): the ranks split int8 products the way the benchmark splits them
across GPUs (column shards with every per-column operand sliced, batch shards with B shared), compute their shards
with the oracle, gather them, and must reproduce the whole product bit for bit. Times combine as the maximum over
ranks. A rank that leaves before a barrier is detected on the host by the other rank's bounded barrier."""
import datetime
import os
import socket

import numpy as np
import pytest

WORLD = 2

CASES = [
    # Ragged N with 256-column shard edges: rank 0 takes 512 columns, rank 1 the remaining 488.
    dict(name="columns-ragged", mode="columns", m=37, n=1000, k=70, batch=1, a_signed=False, b_signed=True,
         za=True, za_vector=False, zb=True, zb_vector=True, transpose_b=False, b_batched=False, align=256),
    # Transposed, batched B (N x K per batch) with per-row zero points of A, 16-column shard edges.
    dict(name="columns-transposed-batched", mode="columns", m=20, n=300, k=33, batch=3, a_signed=True, b_signed=False,
         za=True, za_vector=True, zb=True, zb_vector=False, transpose_b=True, b_batched=True, align=16),
    # Fewer tiles than ranks: rank 1's shard is empty and it still takes part in every collective.
    dict(name="columns-empty-rank", mode="columns", m=9, n=200, k=31, batch=1, a_signed=True, b_signed=True,
         za=False, za_vector=False, zb=True, zb_vector=True, transpose_b=False, b_batched=False, align=256),
    # Batch shards of a product whose batches share B (the batched QKV projection): 3 + 2 batches.
    dict(name="batches-shared-b", mode="batches", m=19, n=48, k=40, batch=5, a_signed=False, b_signed=True,
         za=True, za_vector=False, zb=True, zb_vector=True, transpose_b=False, b_batched=False, align=1),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(case):
    import og_oracle as orc

    m, n, k, batch = case["m"], case["n"], case["k"], case["batch"]
    a = orc.bytes_(batch * m * k, 11).reshape(batch, m, k)
    nb = batch if case["b_batched"] else 1
    b_shape = (nb, n, k) if case["transpose_b"] else (nb, k, n)
    b = orc.bytes_(int(np.prod(b_shape)), 12).reshape(b_shape)
    za = orc.bytes_(m if case["za_vector"] else 1, 13) if case["za"] else None
    zb = orc.bytes_(n if case["zb_vector"] else 1, 14) if case["zb"] else None
    return a, b, za, zb


def _product(case, a, b, za, zb, m, n, batch):
    """The oracle product of already-cut operands: A [batch, m, k], B [nb, k, n] or [nb, n, k]."""
    import og_oracle as orc

    k = case["k"]
    if n == 0 or batch == 0:
        return np.zeros((batch, m, n), np.int32)
    nb = b.shape[0]
    out = orc.int8_gemm(a.reshape(-1), case["a_signed"], b.reshape(-1), case["b_signed"], za, case["za_vector"], zb,
                        case["zb_vector"], threads=1, m=m, n=n, k=k, batch=batch, transpose_b=case["transpose_b"],
                        stride_a=m * k if batch > 1 else 0, stride_b=n * k if nb > 1 else 0)
    return out.reshape(batch, m, n)


def _rank_shard_products(rank, world, port):
    import torch.distributed as dist

    from onegpu_cuda import shard as sh

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=60))
    try:
        for case in CASES:
            a, b, za, zb = _inputs(case)
            m, n, batch = case["m"], case["n"], case["batch"]
            if case["mode"] == "columns":
                s = sh.shard_of(n, world, rank, case["align"])
                b_part = sh.column_slab(b, s, case["transpose_b"])
                zb_part = sh.column_vector(zb, s) if case["zb_vector"] else zb
                part = _product(case, a, b_part, za, zb_part, m, s.width, batch)
            else:
                s = sh.shard_of(batch, world, rank, case["align"])
                a_part = sh.batch_slab(a, s)
                b_part = sh.batch_slab(b, s) if case["b_batched"] else b
                part = _product(case, a_part, b_part, za, zb, m, n, s.width)
            parts = [None] * world
            dist.all_gather_object(parts, part)
            if rank == 0:
                whole = sh.gather_columns(parts) if case["mode"] == "columns" else sh.gather_batches(parts)
                want = _product(case, a, b, za, zb, m, n, batch)
                assert whole.shape == want.shape, case["name"]
                assert np.array_equal(whole, want), case["name"]
        # Times (and any per-rank figure) are reported as the maximum over ranks.
        got = sh.max_over_ranks(dist, [1.5 + rank, -float(rank), 7.0])
        assert got == [0.5 + world, 0.0, 7.0]
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _rank_leaves_early(rank, world, port):
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=30))
    if rank != 0:
        return  # leaves between steps, with nothing in flight
    try:
        dist.monitored_barrier(timeout=datetime.timedelta(seconds=2))
    except RuntimeError as exc:
        assert "1" in str(exc)
    else:
        raise AssertionError("the barrier did not notice that rank 1 had left")


def _spawn(fn):
    import torch.multiprocessing as mp

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    mp.spawn(fn, args=(WORLD, _free_port()), nprocs=WORLD, join=True)


def test_split_covers_the_extent():
    from onegpu_cuda import shard as sh

    for extent in (0, 1, 255, 256, 1000, 8192, 28672):
        for world in (1, 2, 3, 4, 8):
            for align in (1, 16, 256):
                shards = sh.split(extent, world, align)
                assert [s.rank for s in shards] == list(range(world))
                assert shards[0].start == 0 and shards[-1].stop == extent
                for s, t in zip(shards, shards[1:]):
                    assert s.stop == t.start and s.width >= 0
                nonempty = [s for s in shards if s.width > 0]
                assert all(s.start % align == 0 for s in nonempty)
                assert all(s.width % align == 0 for s in nonempty[:-1])  # only the last shard may end ragged
    assert [s.width for s in sh.split(8192, 8, 256)] == [1024] * 8
    assert [s.width for s in sh.split(28672, 8, 256)] == [3584] * 8
    assert [s.width for s in sh.split(1000, 2, 256)] == [512, 488]
    assert [s.width for s in sh.split(200, 2, 256)] == [200, 0]
    with pytest.raises(ValueError):
        sh.shard_of(10, 2, 2)


@pytest.mark.timeout(240)
def test_sharded_products_gather_to_the_whole_product():
    _spawn(_rank_shard_products)


@pytest.mark.timeout(120)
def test_a_rank_that_leaves_is_detected_on_the_host():
    _spawn(_rank_leaves_early)
