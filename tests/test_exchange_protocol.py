"""The slot protocol of the peer-memory exchanges (exchange_kernel in csrc/comm_p2p.cu),
restated on the host: within one call, every word a rank waits for is written exactly once,
no two writes of the call share a slot, and every slot index stays inside its row of
max_elems words. Checked for the one-trip all-reduce and the two-trip form (each slice
sent to its owner rank, summed there, the sums sent back) at 1 to 8 ranks and sizes that do
not divide evenly."""
from collections import Counter

import pytest


def _one_trip(world, n):
    """(writes, waits): writes as (dest rank, source slot, index), waits as (rank, source
    slot, index)."""
    writes = [(r, src, i) for src in range(world) for r in range(world) for i in range(n)]
    waits = [(r, src, i) for r in range(world) for src in range(world) for i in range(n)]
    return writes, waits


def _two_trips(world, n):
    npr = (n + world - 1) // world
    writes, waits = [], []
    # trip 1: rank src sends element i of slice s to the owner s, slot src
    for src in range(world):
        for s in range(world):
            for j in range(npr):
                i = s * npr + j
                if i < n:
                    writes.append((s, src, i))
    # the owner waits for every source of its slice, then sends each sum to the other
    # ranks into its own slot (source = owner)
    for s in range(world):
        for j in range(npr):
            i = s * npr + j
            if i >= n:
                continue
            for src in range(world):
                waits.append((s, src, i))
            for r in range(world):
                if r != s:
                    writes.append((r, s, i))
    # trip 2: rank r waits for the owners' sums of the other slices
    for r in range(world):
        for s in range(world):
            if s == r:
                continue
            for j in range(npr):
                i = s * npr + j
                if i < n:
                    waits.append((r, s, i))
    return writes, waits


@pytest.mark.parametrize("world", range(1, 9))
@pytest.mark.parametrize("n", [1, 7, 64, 1000, 3077])
@pytest.mark.parametrize("form", ["one_trip", "two_trips"])
def test_each_awaited_word_written_once(world, n, form):
    max_elems = (n + 3) // 4 * 4  # rrr_comm_create rounds max_elems up to a multiple of 4
    writes, waits = (_one_trip if form == "one_trip" else _two_trips)(world, n)
    counts = Counter(writes)
    assert max(counts.values()) == 1, "two writes of one call share a slot"
    for w in waits:
        assert counts[w] == 1, w
    for _, src, i in writes:
        assert 0 <= src < world and 0 <= i < max_elems
    if form == "two_trips":
        # every element's sum reaches every rank: each (rank, element) is either owned
        # (summed locally) or awaited once from its owner
        npr = (n + world - 1) // world
        got = Counter((r, i) for r, s, i in waits if s == i // npr and s != r)
        for r in range(world):
            for i in range(n):
                owner = i // npr
                assert (owner == r) != (got[(r, i)] == 1), (r, i)


# ---------------------------------------------------------------- epochs across calls
MAX_CTAS = 64  # kMaxCtas in csrc/comm_p2p.cu


def _chunk(span):
    """Elements per CTA (comm_launch): about 2 KB per rank, at most MAX_CTAS CTAs."""
    c = max(512, (span + MAX_CTAS - 1) // MAX_CTAS)
    return (c + 3) // 4 * 4


def _cta_of(kind, n, world):
    """Element index -> CTA of one call: the one-trip forms map by index, the two-trip
    form by position inside the slice."""
    if kind == "two_trips":
        npr = (n + world - 1) // world
        c = _chunk(npr)
        return lambda i: (i % npr) // c
    c = _chunk(n)
    return lambda i: i // c


def _sets_per_call(calls, world, all_ctas):
    """For each call, element index -> slot set (epoch parity) its words use, with every
    call running all MAX_CTAS CTAs (all_ctas) or only the CTAs that hold data."""
    counters = [0] * MAX_CTAS
    out = []
    for kind, n in calls:
        cta = _cta_of(kind, n, world)
        used = {cta(i) for i in range(n)}
        epoch = {c: counters[c] + 1 for c in range(MAX_CTAS)}
        out.append({i: epoch[cta(i)] & 1 for i in range(n)})
        for c in range(MAX_CTAS):
            if all_ctas or c in used:
                counters[c] += 1
    return out


# the batched decode step's exchanges at 8 ranks: all-reduces of 64 x 3072 (two trips), a
# one-trip exchange of 3072, the logits all-gather rows (64 x 25008 per rank)
STEP = [("two_trips", 64 * 3072), ("two_trips", 64 * 3072), ("one_trip", 3072),
        ("one_trip", 64 * 25008), ("two_trips", 64 * 3072), ("one_trip", 3072)]


def _alternates(sets):
    for a, b in zip(sets, sets[1:]):
        for i in a.keys() & b.keys():
            if a[i] == b[i]:
                return False
    return True


def test_consecutive_calls_use_different_slot_sets():
    """A rank may be one call ahead of another, so consecutive calls must write every
    word they share into different slot sets (the reader of the older call would see the
    newer epoch and wait until its limit). Running all CTAs in every call advances every
    CTA's epoch together, which keeps that however calls of different sizes map elements
    to CTAs; running only the CTAs that hold data does not."""
    assert _alternates(_sets_per_call(STEP, 8, all_ctas=True))
    assert not _alternates(_sets_per_call(STEP, 8, all_ctas=False))
