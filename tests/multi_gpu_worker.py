"""Rank bodies of the multi-GPU tests: each runs in its own spawned process on its own GPU (one process per GPU, as
the library is used across a node). Rank 0 makes the communicator id and hands it to the others through a queue."""
from __future__ import annotations

import traceback

import numpy as np


def gather_rank(rank: int, nranks: int, id_queues, results, m: int, n: int, k: int, seed: int) -> None:
    try:
        import og_oracle as oracle
        import onegpu_cuda as og
        from onegpu_cuda import shard as sh

        if rank == 0:
            uid = og.comm_unique_id()
            for q in id_queues[1:]:
                q.put(uid)
        else:
            uid = id_queues[rank].get(timeout=120)
        with og.GpuDevice(rank) as dev, og.Communicator(dev, nranks, rank, uid) as comm:
            # Every rank draws the whole operands from one seed and keeps its shard, as a caller with replicated
            # activations and column-sharded weights would hold them.
            a = oracle.bytes_(m * k, seed)
            b = oracle.bytes_(k * n, seed + 1).reshape(k, n)
            za = np.array([129], np.uint8)
            zb = oracle.bytes_(n, seed + 2)
            shards = sh.split(n, nranks, sh.TILE_COLUMNS)
            part = shards[rank]
            bslab = sh.column_slab(b, part)
            widths = [s.width for s in shards]
            ba = dev.create_buffer(np.uint8, a)
            bb = dev.create_buffer(np.int8, bslab.view(np.int8).reshape(-1))
            bza = dev.create_buffer(np.uint8, za)
            bzb = dev.create_buffer(np.int8, sh.column_vector(zb, part).view(np.int8))
            bc = dev.create_buffer(np.int32, m * part.width)
            full = dev.create_buffer(np.int32, m * n) if rank == 0 else None
            with og.Int8Gemm(dev) as gemm:
                enc = dev.begin_commands()
                gemm.encode_int32(enc, og.Int8GemmProblem(m, part.width, k), ba, bb, bc, og.Int8Operand(bza, 0),
                                  og.Int8Operand(bzb, 0, True))
                kernel = gemm.last_kernel
                dev.submit(enc)
                comm.gather_columns(bc.ptr, 4, 1, m, widths, full.ptr if full is not None else 0, root=0)
                # The operand replicated the other way: each rank holds one part of A, all_gather gives all of A.
                rows = m // nranks
                mine = dev.create_buffer(np.uint8, a[rank * rows * k:(rank + 1) * rows * k])
                everything = dev.create_buffer(np.uint8, nranks * rows * k)
                comm.all_gather(mine.ptr, rows * k, everything.ptr)
                dev.wait_idle()
                replicated_ok = bool(np.array_equal(everything.read(), a[:nranks * rows * k]))
            out = {"rank": rank, "replicated_ok": replicated_ok, "kernel": kernel}
            if rank == 0:
                got = full.read()
                want = oracle.int8_gemm(a, False, b.reshape(-1), True, za, False, zb, True, m=m, n=n, k=k)
                out["mismatches"] = int(np.count_nonzero(got != want))
            results.put(out)
    except Exception:  # noqa: BLE001 - reported to the parent
        results.put({"rank": rank, "error": traceback.format_exc()})
