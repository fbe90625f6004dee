"""Frame sharding across GPUs: one process per GPU, no collective on the data path.

Frames (SPAN) and frame pairs (RIFE) are independent, so a stream is cut into contiguous chunks
dealt round-robin over the ranks. A chunk also carries the first frame of the next chunk, so
that its last interpolated pair (frame i, frame i + 1) needs no frame from another rank. That one
frame is upscaled twice, once by each of the two ranks: about 2 % redundant work at 48-frame
chunks. Outputs are gathered to the host in chunk order. The only collectives are the timing
barrier and the max-over-ranks of the elapsed time.
"""
from __future__ import annotations

from dataclasses import dataclass

CHAIN_CHUNK = 48  # frames per chunk of the full-chain workload


@dataclass(frozen=True)
class Chunk:
    index: int   # chunk number in the stream
    first: int   # first frame of the chunk
    last: int    # one past the last frame the chunk owns
    upto: int    # one past the last frame the chunk reads (last + 1 except at the end of the stream)

    @property
    def pairs(self):
        """(i, i + 1) frame pairs this chunk interpolates."""
        return [(i, i + 1) for i in range(self.first, self.upto - 1)]


def chunks_for_rank(n_frames: int, world: int, rank: int, chunk: int = CHAIN_CHUNK) -> list[Chunk]:
    """Contiguous chunks of `chunk` frames, chunk c to rank c % world."""
    if world < 1 or not 0 <= rank < world or chunk < 1 or n_frames < 0:
        raise ValueError("bad shard request")
    out = []
    for c in range(rank, -(-n_frames // chunk), world):
        first = c * chunk
        last = min(n_frames, first + chunk)
        out.append(Chunk(c, first, last, min(n_frames, last + 1)))
    return out


def frame_seed(base: int, rank: int, i: int) -> int:
    """Seed of the i-th synthetic frame of a rank: distinct across ranks and frames."""
    return base + 100003 * rank + i


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank number over all ranks (the timing rule: a multi-GPU time is the slowest
    rank's). Works on the nccl and gloo backends; returns the value itself without a process group."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(device=None) -> None:
    """A barrier that also works where dist.barrier() would need a device (one all-reduce)."""
    import torch
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.ones(1, device=device)
        dist.all_reduce(t)
    if device is not None and str(device).startswith("cuda"):
        torch.cuda.synchronize()


def whole_job_rate(units_per_rank: int, world: int, seconds_max: float) -> float:
    """Units per second over all ranks: every rank processes units_per_rank in at most seconds_max."""
    if seconds_max <= 0:
        raise ValueError("elapsed time must be positive")
    return units_per_rank * world / seconds_max
