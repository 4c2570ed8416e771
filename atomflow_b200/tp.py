"""Megatron-style tensor-parallel split of the decode projections.

Column-parallel projections (fused QKV, gate, up) split the output rows N;
row-parallel ones (O, down) split K and need a sum (all-reduce) of the
partial outputs.  K / world stays a multiple of 128 for every shape used here
(3072/8 = 384, 8192/8 = 1024, 4096/8 = 512, 14336/8 = 1792), so the 128-wide
scale groups of a K shard are exactly the full matrix's groups: quantising a
shard gives the same bytes and scales as slicing the quantised matrix.
"""


def shard(w, x, split, rank, world):
    """(w [N, K], x [M, K]) -> this rank's (w, x).  split: 'col' or 'row'."""
    if world == 1:
        return w, x
    if split == "col":
        n = w.shape[0]
        if n % world:
            raise ValueError(f"N={n} is not divisible by world={world}")
        return w.chunk(world, 0)[rank], x
    k = w.shape[1]
    if k % (128 * world):
        raise ValueError(f"K={k} must split into multiples of 128 over {world} ranks")
    return w.chunk(world, 1)[rank], x.chunk(world, x.dim() - 1)[rank]
