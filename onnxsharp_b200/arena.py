"""Device-memory arena for a static plan: the reference's lifetime colouring
with byte offsets in one device buffer instead of grow-only slot objects.

Reference: ``BufferAllocator.Assign`` (src/OnnxSharp/Engine/BufferAllocator.cs:41-138)
— buffers ordered by first write (ties by index), each takes the slot whose
previous occupant's last read is the latest one strictly before this
buffer's first write (strict ``<``: a slot read by an op is never rewritten
by the same op), else a new slot; an in-place output (``inplace[dst] = src``)
shares its source's slot and extends its lifetime. A slot's size is the
largest of its buffers; slots are laid out back to back, 256-byte aligned.
"""
from __future__ import annotations

from dataclasses import dataclass

ALIGN = 256
NO_SLOT = -1


@dataclass(frozen=True)
class Lifetime:
    first_write: int  # op index of the first write
    last_read: int    # op index of the last read (graph outputs: len(prog))
    nbytes: int


def assign_slots(lifetimes: list[Lifetime], inplace: dict[int, int] | None = None) -> tuple[list[int], int]:
    """Slot index per buffer (NO_SLOT if never written) and the slot count."""
    inplace = inplace or {}
    slot_of = [NO_SLOT] * len(lifetimes)
    order = sorted((i for i, lt in enumerate(lifetimes) if lt.first_write >= 0),
                   key=lambda i: (lifetimes[i].first_write, i))
    free_at: list[int] = []
    for i in order:
        start = lifetimes[i].first_write
        end = max(lifetimes[i].last_read, start)
        src = inplace.get(i, -1)
        if src >= 0 and slot_of[src] >= 0:
            s = slot_of[src]
            slot_of[i] = s
            free_at[s] = max(free_at[s], end)
            continue
        chosen, best = NO_SLOT, None
        for s, f in enumerate(free_at):
            if f < start and (best is None or f > best):
                best, chosen = f, s
        if chosen == NO_SLOT:
            chosen = len(free_at)
            free_at.append(end)
        else:
            free_at[chosen] = end
        slot_of[i] = chosen
    return slot_of, len(free_at)


def plan_offsets(lifetimes: list[Lifetime], inplace: dict[int, int] | None = None) -> tuple[list[int], int]:
    """Byte offset per buffer (-1 if never written) and the arena size."""
    slot_of, nslots = assign_slots(lifetimes, inplace)
    size = [0] * nslots
    for i, s in enumerate(slot_of):
        if s >= 0:
            size[s] = max(size[s], lifetimes[i].nbytes)
    base, off = [0] * nslots, 0
    for s in range(nslots):
        base[s] = off
        off += (size[s] + ALIGN - 1) // ALIGN * ALIGN
    return [base[s] if s >= 0 else -1 for s in slot_of], off


def plan_offsets_dag(lifetimes: list[Lifetime], touch: list[int], anc: list[int]) -> tuple[list[int], int]:
    """plan_offsets for a plan whose nodes may run concurrently on several
    streams. touch[i] is a bitmask of the node indices that read or write
    buffer i; anc[n] a bitmask of the nodes that happen before node n (data
    dependencies and earlier nodes on n's stream). A slot is reused under the
    reference's rule AND only when every node that touched its earlier
    occupants happens before the new buffer's first writer, so no buffer is
    overwritten while a concurrent branch may still read it. With one stream
    every earlier node happens before, and this is plan_offsets exactly."""
    slot_of = [NO_SLOT] * len(lifetimes)
    order = sorted((i for i, lt in enumerate(lifetimes) if lt.first_write >= 0),
                   key=lambda i: (lifetimes[i].first_write, i))
    free_at: list[int] = []
    slot_touch: list[int] = []
    for i in order:
        start = lifetimes[i].first_write
        end = max(lifetimes[i].last_read, start)
        chosen, best = NO_SLOT, None
        for s, f in enumerate(free_at):
            if f < start and (slot_touch[s] & ~anc[start]) == 0 and (best is None or f > best):
                best, chosen = f, s
        if chosen == NO_SLOT:
            chosen = len(free_at)
            free_at.append(end)
            slot_touch.append(touch[i])
        else:
            free_at[chosen] = end
            slot_touch[chosen] |= touch[i]
        slot_of[i] = chosen
    size = [0] * len(free_at)
    for i, s in enumerate(slot_of):
        if s >= 0:
            size[s] = max(size[s], lifetimes[i].nbytes)
    base, off = [0] * len(free_at), 0
    for s in range(len(free_at)):
        base[s] = off
        off += (size[s] + ALIGN - 1) // ALIGN * ALIGN
    return [base[s] if s >= 0 else -1 for s in slot_of], off
