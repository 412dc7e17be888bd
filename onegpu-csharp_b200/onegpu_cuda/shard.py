"""How one int8 product is divided among ranks (one process per GPU) and put back together.

The product has no reduction across ranks: every output element needs one row of A and one column of B only. So G
ranks split it with no exchange in the data path:

* column shards: rank g computes C[:, :, n0:n0+w] from the full A and its slab of B's columns (a contiguous
  K x w array, bound with Ldb = w, or the w rows of a transposed B); every per-column operand (zero points of B,
  scales, biases) is sliced the same way;
* batch shards: rank g computes batches [b0, b0+w) of a batched product from its batches of A (and of B when B is
  batched); B is replicated when every batch shares it.

Shard edges are multiples of ``align`` units (the product's 256-column tile by default) so that no output tile
straddles two ranks; the first ranks take one unit more when the units do not divide evenly, the last unit may be
partial, and ranks beyond the work get empty shards. Putting C back together is a concatenation along the split
axis (``gather_columns`` / ``gather_batches``), and times are combined as the maximum over ranks
(``max_over_ranks``), the figure a multi-GPU step is reported with.

The reference runs every device on its own, with no cross-device traffic (MultiDeviceTests.cs:6-107), so this module
has no counterpart there.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np

TILE_COLUMNS = 256  # columns of one output tile of the tensor-core product


@dataclass(frozen=True)
class Shard:
    rank: int
    start: int
    width: int

    @property
    def stop(self) -> int:
        return self.start + self.width


def split(extent: int, world: int, align: int = 1) -> list[Shard]:
    """The shards of ``extent`` units among ``world`` ranks, edges on multiples of ``align``."""
    if world < 1:
        raise ValueError("world must be at least 1")
    if extent < 0 or align < 1:
        raise ValueError("extent must be non-negative and align positive")
    units = -(-extent // align)
    base, extra = divmod(units, world)
    shards = []
    start = 0
    for g in range(world):
        width = min((base + (1 if g < extra else 0)) * align, extent - start)
        shards.append(Shard(g, start, width))
        start += width
    return shards


def shard_of(extent: int, world: int, rank: int, align: int = 1) -> Shard:
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return split(extent, world, align)[rank]


def column_slab(b: np.ndarray, shard: Shard, transpose_b: bool = False) -> np.ndarray:
    """The contiguous slab of B for a column shard. ``b`` is [..., K, N] (or [..., N, K] when transposed)."""
    if transpose_b:
        return np.ascontiguousarray(b[..., shard.start:shard.stop, :])
    return np.ascontiguousarray(b[..., :, shard.start:shard.stop])


def column_vector(v: np.ndarray | None, shard: Shard) -> np.ndarray | None:
    """A per-column operand (zero points of B, scales, biases) cut to a column shard; scalars pass through."""
    if v is None or np.ndim(v) == 0 or np.size(v) == 1:
        return v
    return np.ascontiguousarray(v[shard.start:shard.stop])


def batch_slab(x: np.ndarray, shard: Shard) -> np.ndarray:
    """Batches [start, stop) of a batched operand [batch, ...]."""
    return np.ascontiguousarray(x[shard.start:shard.stop])


def gather_columns(parts: Sequence[np.ndarray]) -> np.ndarray:
    """C from its column shards, each [..., M, w_g], in rank order."""
    return np.concatenate(list(parts), axis=-1)


def gather_batches(parts: Sequence[np.ndarray]) -> np.ndarray:
    """C from its batch shards, each [w_g, M, N], in rank order."""
    return np.concatenate(list(parts), axis=0)


def max_over_ranks(dist, values: Sequence[float], device=None) -> list[float]:
    """The element-wise maximum of ``values`` over all ranks of the default process group (``dist`` is
    torch.distributed; ``device`` is the rank's CUDA device under NCCL, None under gloo)."""
    import torch

    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.cpu().tolist()]
