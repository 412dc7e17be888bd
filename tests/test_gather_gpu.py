"""Gathering N-sharded results over NVLink (og_comm_gather_columns) and replicating an operand (og_comm_all_gather),
two GPUs, one spawned process each, against the oracle bit for bit. Runs where at least two GPUs are visible (the
multi-GPU calls of the build); a single-GPU run skips it."""
import multiprocessing as mp

import pytest

import onegpu_cuda as og
from multi_gpu_worker import gather_rank

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(1000, 2048 + 512, 768), (8192, 2048, 8192)])
def test_column_shards_gathered_onto_one_gpu_are_bit_exact(m, n, k):
    if og.device_count() < 2:
        pytest.skip("needs two GPUs")
    nranks = 2
    ctx = mp.get_context("spawn")  # a fresh CUDA context per rank
    id_queues = [ctx.Queue() for _ in range(nranks)]
    results = ctx.Queue()
    procs = [ctx.Process(target=gather_rank, args=(r, nranks, id_queues, results, m, n, k, 11 + m % 7))
             for r in range(nranks)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(nranks):
            r = results.get(timeout=300)
            got[r["rank"]] = r
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in got.values():
        assert "error" not in r, r.get("error")
        assert r["replicated_ok"], r
    assert got[0]["mismatches"] == 0
