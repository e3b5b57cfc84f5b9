"""Batch sharding of independent sequences over the GPUs of one node.

Sequences never interact on TextEngine's path, so N GPUs decode N contiguous blocks of rows with
no collective on the data path; ``torch.distributed`` only carries start/stop barriers, timing
and the final gather of tokens.

Sampling must not depend on the split. TextEngine draws one ``nextDouble`` (two generator steps)
per token from one engine-wide java.util.Random (TextEngine.java:43,417). Decoding rows one after
another from a single seed therefore starts row r at the seeded state advanced by 2*steps*r. A
shard that begins at global row ``first`` sets its engine generator to that state
(``bst_set_rng_state``); its rows then draw exactly what the unsharded run draws.
"""
from __future__ import annotations

MULTIPLIER = 0x5DEECE66D
ADDEND = 0xB
MASK = (1 << 48) - 1


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s contiguous shard; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(total, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def scramble(seed: int) -> int:
    """java.util.Random.setSeed: the generator state a seed produces."""
    return (seed ^ MULTIPLIER) & MASK


def advance(state: int, steps: int) -> int:
    """The generator state `steps` LCG steps after `state`, by squaring the affine map."""
    mul, add = 1, 0
    step_mul, step_add = MULTIPLIER, ADDEND
    while steps:
        if steps & 1:
            mul = (mul * step_mul) & MASK
            add = (add * step_mul + step_add) & MASK
        step_add = (step_add * step_mul + step_add) & MASK
        step_mul = (step_mul * step_mul) & MASK
        steps >>= 1
    return (state * mul + add) & MASK


def shard_rng_state(seed: int, steps: int, first_row: int) -> int:
    """Generator state for a shard whose first global row is `first_row`, when the unsharded run
    seeds once with `seed` and samples `steps` tokens per row, row after row."""
    return advance(scramble(seed), 2 * steps * first_row)
