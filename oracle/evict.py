"""Rolling-window (attention sinks) eviction schedule -- restated from the engine.

``src/engine.ts:1188-1214``: when a batch of ``n`` new rows would overflow ``maxSeqLen``
(``evictFor``), the engine frees ``need = fill + n - maxSeqLen`` slots plus a quarter-window
batch::

    recent = fill - SINKS
    batch  = min(recent, max(need, ceil((maxSeqLen - SINKS) / 4)))
    keep   = recent - batch
    if keep <= 0: return SINKS                 # sinks only
    move rows [SINKS + batch, fill) down to [SINKS, SINKS + keep)
    return SINKS + keep

The cache bytes only move (no re-rope, no requantise); attention rotates K by the new slot
index at read.  ``LogicalWindow`` replays that schedule on a list of logical token ids so
tests can ask "which token sits in slot j" after any number of evictions, independently of
the physical ring the B200 cache uses.
"""
import math


def evict_plan(fill, need, sinks, max_seq_len):
    """Returns ``(batch, new_fill)`` exactly as ``engine.ts:1188-1194,1210``."""
    recent = fill - sinks
    batch = min(recent, max(need, math.ceil((max_seq_len - sinks) / 4)))
    keep = recent - batch
    if keep <= 0:
        return recent, sinks
    return batch, sinks + keep


def evict_for(fill, n, sinks, max_seq_len):
    """``engine.ts:1214``: evict only when ``fill + n > maxSeqLen``.  Returns
    ``(batch_evicted, new_fill)`` (batch 0 when nothing happens)."""
    if fill + n > max_seq_len:
        return evict_plan(fill, fill + n - max_seq_len, sinks, max_seq_len)
    return 0, fill


class LogicalWindow:
    """Logical slot contents (token ids) under the reference's compaction schedule."""

    def __init__(self, sinks, max_seq_len):
        self.sinks = sinks
        self.max = max_seq_len
        self.slots = []          # slot j -> token id

    @property
    def fill(self):
        return len(self.slots)

    def append(self, tokens):
        tokens = list(tokens)
        batch, new_fill = evict_for(self.fill, len(tokens), self.sinks, self.max)
        if batch:
            keep = new_fill - self.sinks
            self.slots = self.slots[:self.sinks] + self.slots[self.fill - keep:]
        start = self.fill
        self.slots.extend(tokens)
        return batch, start
