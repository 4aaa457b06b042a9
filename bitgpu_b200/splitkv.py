"""Split-KV decode across GPUs for one long stream (config 5b: the 27B hybrid's gated head_dim-256
attention at 131072 positions).

The reference is single-device; this is the B200 extension for a stream whose cache is spread
over the ranks of one node.  Rank r holds the contiguous slice of cache positions
``[lo_r, hi_r)`` (``split_bounds``).  Every step:

1. each rank runs ``bg_attention_partials`` over its slice and produces rows of
   ``(unnormalised o[D], m, l)``;
2. one NCCL all-gather over NVLink brings every rank's partial rows into local memory;
3. every rank merges the partials by log-sum-exp with ``bg_lse_merge``, with the sigmoid output
   gate fused into the merge.

The payload is ``H*(D+2)*4`` bytes per rank per query row (24.8 KB for 24 heads of 256).  No kernel
reads peer memory.

``partials_fn`` / ``merge_fn`` default to the CUDA entry points.  The CPU tests substitute the
oracle, so the collective orchestration runs on ``gloo`` ranks without a GPU.
"""
import torch
import torch.distributed as dist


class PeerFailure(RuntimeError):
    """The exchange of one step did not complete: a rank left (raised, exited, or never joined
    the step) and the collective ended with an error or ran into the process group's timeout.
    The surviving ranks raise this instead of waiting forever; the stream's output for that step
    does not exist."""


def split_bounds(L, world):
    """Contiguous, near-equal slices of ``L`` positions over ``world`` ranks:
    ``[(lo, hi), ...]``; the first ``L % world`` ranks take one extra position."""
    base, extra = divmod(L, world)
    out, lo = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((lo, lo + n))
        lo += n
    return out


def _cuda_partials(q, local_cache, pos_base, lo, hi, scale):
    from . import ops
    return ops.attention_partials(q, local_cache, pos_base, lo, hi, scale=scale)


def _cuda_merge(gathered, out_shape, gate):
    from . import ops
    return ops.lse_merge(gathered, out_shape, gate=gate)


class SplitKVDecoder:
    """One rank's view of a stream whose KV positions are sharded over ``group``."""

    def __init__(self, L, group=None, partials_fn=None, merge_fn=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.bounds = split_bounds(L, self.world)
        self.lo, self.hi = self.bounds[self.rank]
        self.partials_fn = partials_fn or _cuda_partials
        self.merge_fn = merge_fn or _cuda_merge

    def step(self, q, local_cache, pos_base, gate=None, scale=0.0):
        """``q[B, S, H, D]`` (replicated on every rank) -> gated attention output ``[B, S, H, D]``
        over all ranks' positions ``0 .. pos_base+qi``."""
        B, S, H, D = q.shape
        hi = max(self.lo, min(self.hi, pos_base + S))  # a slice past the last position is empty
        part = self.partials_fn(q, local_cache, pos_base, self.lo, hi, scale)
        if self.world == 1:
            gathered = part.unsqueeze(0)
        else:
            rows, w = part.shape
            flat = torch.empty((self.world * rows, w), dtype=part.dtype, device=part.device)
            try:
                dist.all_gather_into_tensor(flat, part.contiguous(), group=self.group)
            except (RuntimeError, dist.DistError) as e:  # peer gone or timed out
                raise PeerFailure(f"split-KV exchange failed on rank {self.rank} of {self.world}: {e}") from e
            gathered = flat.view(self.world, rows, w)
        return self.merge_fn(gathered, (B, S, H, D), gate)
