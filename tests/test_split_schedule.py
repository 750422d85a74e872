"""Properties of the decode GEMV's stream-K schedule that its split-unit reduction relies on (b70-inference_b200/csrc/
gemv.cuh: range_start / owner_of / next_owner, the partial-slot choice and the first-contributor finisher), checked
on the host over many launch shapes. The formulas are restated here; the GPU tests check the kernels' results.

* The contributors of a unit, enumerated from the owner of its first k-block by next_owner, are exactly the CTAs
  whose ranges intersect it, in CTA order.
* A contributor's partial slot (2c for the first segment of its range, 2c + 1 otherwise) is the one the finisher
  reads (2c + 1 when its range starts before the unit, else 2c).
* A split unit is the last segment of its first contributor's range (that CTA finishes it after its own part).
* A CTA has at most one segment that is a split unit it does not finish, and it is the first segment of its range
  (the one ticket a CTA reads at the end of the launch)."""
import pytest


def range_start(c, T, G):
    return c * T // G


def owner_of(x, T, G):
    return ((x + 1) * G - 1) // T


def next_owner(c, T, G):
    return owner_of(range_start(c + 1, T, G), T, G)


def segments(c, T, G, KB):
    """The units CTA c's range touches, in order: (unit, lo, hi) in k-blocks of the unit."""
    r0, r1 = range_start(c, T, G), range_start(c + 1, T, G)
    if r1 <= r0:
        return []
    u0 = r0 // KB
    out = []
    for u in range(u0, (r1 - 1) // KB + 1):
        lo = r0 - u * KB if u == u0 else 0
        hi = min(KB, r1 - u * KB)
        out.append((u, lo, hi))
    return out


@pytest.mark.parametrize("U,KB", [(1, 1), (2, 8), (3, 5), (160, 16), (640, 4), (200, 40), (7, 128), (40, 3)])
@pytest.mark.parametrize("G", [1, 2, 3, 7, 64, 148])
def test_split_unit_bookkeeping(U, KB, G):
    T = U * KB
    segs = {c: segments(c, T, G, KB) for c in range(G)}
    for u in range(U):
        a0, a1 = u * KB, (u + 1) * KB
        touching = [c for c in range(G) if any(s[0] == u for s in segs[c])]
        # enumeration from the owner of a0
        enum = []
        c = owner_of(a0, T, G)
        while True:
            enum.append(c)
            if range_start(c + 1, T, G) >= a1:
                break
            c = next_owner(c, T, G)
        assert enum == touching, (u, enum, touching)
        if len(enum) == 1:
            continue
        head = enum[0]
        assert segs[head][-1][0] == u, "a split unit is the last segment of its first contributor"
        for c in enum:
            i = [s[0] for s in segs[c]].index(u)
            written = 2 * c if i == 0 else 2 * c + 1
            read = 2 * c + 1 if range_start(c, T, G) < a0 else 2 * c
            assert written == read, (u, c)
    for c in range(G):
        not_finished = []
        for i, (u, lo, hi) in enumerate(segs[c]):
            split = not (lo == 0 and hi == KB)
            if split and owner_of(u * KB, T, G) != c:
                not_finished.append(i)
        assert not_finished in ([], [0]), (c, not_finished)
