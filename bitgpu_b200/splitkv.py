"""Split-KV decode across GPUs for one long stream (config 5b: the 27B hybrid's gated head_dim-256
attention at 131072 positions).

The reference is single-device; this is the B200 extension for a stream whose cache is spread
over the ranks of one node.  Rank r holds the contiguous slice of cache positions
``[lo_r, hi_r)`` (``split_bounds``).  Every step:

1. each rank runs the split-KV partials over its slice and produces rows of
   ``(unnormalised o[D], m, l)``;
2. the rows reach every rank;
3. every rank merges the partials by log-sum-exp, with the sigmoid output gate fused into the
   merge.

Step 2 has two forms:

* ``exchange="peer"`` (default on GPUs): ``bg_attention_peer`` -- the split-KV kernel, then a
  push kernel that merges this rank's splits and stores the rows straight into every rank's
  gather buffer over NVLink (plain peer stores into torch symmetric memory) and counts them on
  every rank, then a merge kernel that waits (bounded) for the other ranks' rows, merges and
  gates.  No collective; the step counter lives on the device, so a step can be captured in a
  CUDA graph.
* ``exchange="nccl"``: ``bg_attention_partials``, one NCCL all-gather, ``bg_lse_merge`` (also the
  form the CPU tests run on ``gloo`` ranks).

The payload is ``H*(D+2)*4`` bytes per rank per query row (24.8 KB for 24 heads of 256).

``partials_fn`` / ``merge_fn`` replace the kernels of the ``nccl`` form: the CPU tests substitute the
oracle, so the collective orchestration runs on ``gloo`` ranks without a GPU.
"""
import torch
import torch.distributed as dist


class PeerFailure(RuntimeError):
    """The exchange of one step did not complete: a rank left (raised, exited, or never joined
    the step) and the collective ended with an error or ran into the process group's timeout.
    The surviving ranks raise this instead of waiting forever; the stream's output for that step
    does not exist."""


class PeerExchange:
    """One rank's side of the peer-memory exchange: a buffer every rank of ``group`` can address
    (torch symmetric memory: gather slots ``[2][nranks][rows][D+2]`` f32, then ``[nranks][rows]`` u32
    arrival counters), this rank's step / merge counters and per-group tickets, and the
    ``bg_peer_exchange`` descriptor that carries every rank's addresses as seen from this GPU."""

    def __init__(self, rows, D, group=None, spin_limit=0):
        import torch.distributed._symmetric_memory as symm_mem
        from ._lib import MAX_PEERS, PeerExchange as Desc, lib
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_PEERS:
            raise ValueError(f"peer exchange supports at most {MAX_PEERS} ranks")
        self.rows, self.D = rows, D
        L = lib()
        nbytes = L.bg_peer_exchange_bytes(self.world, rows, D)
        foff = L.bg_peer_exchange_flags_offset(self.world, rows, D)
        dev = torch.device("cuda", torch.cuda.current_device())
        gname = (group or dist.group.WORLD).group_name
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, gname)
        self.ctr = torch.zeros(2 + rows, dtype=torch.int32, device=dev)  # step, done, tickets (<= rows groups)
        ptrs = list(self.handle.buffer_ptrs)
        self.desc = Desc()
        self.desc.nranks, self.desc.rank = self.world, self.rank
        for r in range(self.world):
            self.desc.gather[r] = ptrs[r]
            self.desc.flags[r] = ptrs[r] + foff
        self.desc.step = self.ctr.data_ptr()
        self.desc.done = self.ctr.data_ptr() + 4
        self.desc.tickets = self.ctr.data_ptr() + 8
        self.desc.spin_limit = spin_limit
        torch.cuda.synchronize()
        dist.barrier(group)  # every rank's buffer is zeroed before anyone pushes


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

    def __init__(self, L, group=None, partials_fn=None, merge_fn=None, exchange="auto", spin_limit=0):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.bounds = split_bounds(L, self.world)
        self.lo, self.hi = self.bounds[self.rank]
        self.partials_fn = partials_fn or _cuda_partials
        self.merge_fn = merge_fn or _cuda_merge
        if exchange == "auto":
            exchange = "peer" if (self.world > 1 and partials_fn is None and merge_fn is None
                                  and dist.get_backend(group) == "nccl") else "nccl"
        if exchange not in ("peer", "nccl"):
            raise ValueError(exchange)
        self.exchange = exchange
        self.spin_limit = spin_limit
        self.px = None

    def close(self):
        """Release the peer buffers collectively (every rank calls it, with no step in flight)
        before the process group goes away."""
        if self.px is not None:
            torch.cuda.synchronize()
            dist.barrier(self.group)
            self.px = None

    def step(self, q, local_cache, pos_base, gate=None, scale=0.0):
        """``q[B, S, H, D]`` (replicated on every rank) -> gated attention output ``[B, S, H, D]``
        over all ranks' positions ``0 .. pos_base+qi``."""
        B, S, H, D = q.shape
        hi = max(self.lo, min(self.hi, pos_base + S))  # a slice past the last position is empty
        if self.exchange == "peer" and self.world > 1:
            from . import ops
            rows = B * S * H
            if self.px is None or (self.px.rows, self.px.D) != (rows, D):
                self.px = PeerExchange(rows, D, self.group, self.spin_limit)
            return ops.attention_peer(q, local_cache, pos_base, self.lo, hi, self.px, scale=scale, gate=gate)
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
