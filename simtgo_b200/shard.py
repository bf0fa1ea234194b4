"""How the sharded workloads split across ranks (one process per GPU).

The reference has no multi-GPU support (README.md:64-66); these plans are
the B200 build's. All three are partitions of one long 1-D signal:

  FIR          contiguous output blocks; each shard's input starts `halo`
               samples before its first output (halo >= taps-1), so no
               data-path collective is needed -- the preceding samples are
               duplicated when the shard is placed in HBM.
  Histogram    contiguous sample blocks; per-shard bins summed over ranks.
  tile graph   contiguous element blocks; a halo only if the graph has a
               window (FIR) node.

halo values are rounded up to a multiple of 4 samples so that every shard's
own data starts 16-byte aligned relative to its input buffer.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    out_lo: int    # first global output (or sample) this rank owns
    out_hi: int    # one past the last
    in_lo: int     # first global input sample this rank reads (out_lo - halo)
    halo: int      # samples before out_lo staged with the shard

    @property
    def n(self) -> int:
        return self.out_hi - self.out_lo

    @property
    def in_len(self) -> int:
        return self.out_hi - self.in_lo


def split(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous near-equal blocks; the first total % world ranks get one
    more element."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def round_halo(window: int) -> int:
    """Samples of halo a window of `window` taps needs, rounded up to 4."""
    need = max(0, window - 1)
    return (need + 3) // 4 * 4


def fir_plan(total: int, world: int, rank: int, taps: int) -> Shard:
    lo, hi = split(total, world, rank)
    halo = min(lo, round_halo(taps))
    return Shard(rank, lo, hi, lo - halo, halo)


def histogram_plan(total: int, world: int, rank: int) -> Shard:
    lo, hi = split(total, world, rank)
    return Shard(rank, lo, hi, lo, 0)


def chain_window(taps_along_chain) -> int:
    """The window one FIR of `taps` would need to reach as far below a
    position as a chain of FIRs does (each reads the one inside it, the
    library's opt-in chained windows): 1 + the sum of taps-1 over the chain.
    Pass it as tile_plan's max_taps for a shard that is exact at its edge."""
    return 1 + sum(max(0, int(t) - 1) for t in taps_along_chain)


def tile_plan(total: int, world: int, rank: int, max_taps: int = 0) -> Shard:
    """Contiguous element blocks; with a window (FIR) node of at most
    max_taps taps -- or a chain of them, see chain_window -- each shard's
    inputs start round_halo(max_taps) samples early."""
    lo, hi = split(total, world, rank)
    halo = min(lo, round_halo(max_taps)) if max_taps > 0 else 0
    return Shard(rank, lo, hi, lo - halo, halo)
