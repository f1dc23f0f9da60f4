"""Index arithmetic of the per-token chain kernel (csrc/chain.cu), restated
in Python and checked on the CPU for every linear of the 14B stack at 1, 2,
4 and 8 ranks on 148 CTAs, and for the GPU tests' small links: every item is
owned by exactly one CTA; a row block cut between CTAs gets exactly as many
arrivals as the kernel's owner count expects (CTAs that own no item of a
linear must not be counted), and its finisher reads exactly the slots the
contributors wrote; each CTA's quantised activation range covers the units
its items decode."""
import pytest

ROW_BUDGET = 4400
UB = {4: 144, 5: 176, 6: 210}


def plan(q, K, N, world):
    n = N // world
    units = K // 256
    row_bytes = units * UB[q]
    T = (n + 15) // 16
    if row_bytes <= ROW_BUDGET:  # whole rows (the pitch check only narrows this further)
        S, upi = 1, units
    else:
        upi_max = max(1, ROW_BUDGET // UB[q])
        S = -(-units // upi_max)
        upi = -(-units // S)
    return dict(T=T, S=S, upi=upi, units=units, I=T * S)


def first_item(c, I, G):
    return c * I // G


def cta_of_item(i, I, G):
    return ((i + 1) * G - 1) // I


def check(p, G=148):
    I, S, T, upi, units = p["I"], p["S"], p["T"], p["upi"], p["units"]
    owner = {}
    writes = {}  # (cta, which) -> tile
    arrivals = {}
    for c in range(G):
        i0, i1 = first_item(c, I, G), first_item(c + 1, I, G)
        for i in range(i0, i1):
            assert i not in owner
            owner[i] = c
            assert cta_of_item(i, I, G) == c
        if i1 <= i0:
            continue
        first_tile, last_tile = i0 // S, (i1 - 1) // S
        for tb in range(first_tile, last_tile + 1):
            whole = tb * S >= i0 and (tb + 1) * S <= i1
            if not whole:
                which = 0 if tb == first_tile else 1
                assert (c, which) not in writes
                writes[(c, which)] = tb
                arrivals[tb] = arrivals.get(tb, 0) + 1
        # activation runs quantised by this CTA cover the units its items decode
        all_units = (i1 - i0) >= S or i0 // S != (i1 - 1) // S
        ua = (i0 % S) * upi
        ue = units if S == 1 else min(units, ((i1 - 1) % S + 1) * upi)
        lo, hi = (0, units) if all_units else (ua, ue)
        for i in range(i0, i1):
            u0 = (i % S) * upi
            u1 = min(units, u0 + upi)
            assert lo <= u0 and u1 <= hi
    assert sorted(owner) == list(range(I))
    for tb, got in arrivals.items():
        owners, prev, read = 0, -1, []
        for i in range(tb * S, (tb + 1) * S):
            c = cta_of_item(i, I, G)
            if c != prev:
                owners += 1
                read.append((c, 0 if tb == first_item(c, I, G) // S else 1))
            prev = c
        assert got == owners, (tb, got, owners)
        assert all(writes[r] == tb for r in read) and len(read) == got


STACK = [(4, 5120, 6144), (6, 5120, 1024), (4, 5120, 5120), (4, 5120, 27648), (6, 13824, 5120), (6, 5120, 152064)]
SMALL = [(4, 1024, 768), (6, 1024, 200), (4, 512, 1024), (6, 1024, 512), (5, 512, 8192), (6, 5632, 512),
         (4, 8192, 256)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_stack_links(world):
    for q, K, N in STACK:
        check(plan(q, K, N, world))


@pytest.mark.parametrize("world", [1, 2])
def test_small_links(world):
    for q, K, N in SMALL:
        check(plan(q, K, N, world))


def test_fewer_items_than_ctas_with_split_rows():
    """The case that needs the owner count: 64 items (32 row blocks of 2)
    over 148 CTAs leaves CTAs without items between a block's two owners."""
    p = plan(6, 5632, 512, 1)
    assert p["I"] < 148 and p["S"] == 2
    check(p)
