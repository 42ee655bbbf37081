"""CPU check of the conv kernels' edge-balanced split (conv_tp.cuh: edge_range, row_of_node, cta_of_edge,
finish_pieces), restated in Python: for ragged CSRs (empty nodes, nodes larger than a CTA's range, single-node
graphs), every edge is handled by exactly one CTA, every node's row is written exactly once, and the CTA that finishes
a split node sums exactly the pieces of the CTAs that published one for it, in CTA order."""
import numpy as np
import pytest


def lower_bound(rowptr, n, q):
    lo, hi = 0, n
    while lo < hi:
        mid = (lo + hi) >> 1
        if rowptr[mid] >= q:
            hi = mid
        else:
            lo = mid + 1
    return lo


def edge_range(rowptr, n, E, c, G):
    q0, q1 = E * c // G, E * (c + 1) // G
    lo = lower_bound(rowptr, n, q0)
    n_first = lo - 1 if (lo > 0 and rowptr[lo] > q0) else lo
    n_end = n if c == G - 1 else lower_bound(rowptr, n, q1)
    return q0, q1, n_first, n_end


def cta_of_edge(q, E, G):
    c = q * G // max(E, 1)
    while c + 1 < G and E * (c + 1) // G <= q:
        c += 1
    while c > 0 and E * c // G > q:
        c -= 1
    return c


def simulate(rowptr, G):
    n, E = len(rowptr) - 1, int(rowptr[-1])
    edge_seen = np.zeros(E, int)
    written = np.zeros(n, int)
    published = {}                                  # cta -> node of its part[2c] piece
    pieces = {}                                     # node -> list of ctas that computed a piece
    for c in range(G):
        q0, q1, n_first, n_end = edge_range(rowptr, n, E, c, G)
        for v in range(n_first, n_end):
            p0, p1 = max(rowptr[v], q0), min(rowptr[v + 1], q1)
            edge_seen[p0:p1] += 1
            head, tail = rowptr[v] < q0, rowptr[v + 1] > q1
            if not head and not tail:
                written[v] += 1
            else:
                pieces.setdefault(v, []).append(c)
                if tail:
                    assert c not in published, 'two published pieces in one CTA'
                    published[c] = v
        any_ = n_end > n_first
        if any_ and rowptr[n_first] < q0 and rowptr[n_first + 1] <= q1:          # finalize the first node
            v = n_first
            c_first = cta_of_edge(rowptr[v], E, G)
            assert all(published.get(k) == v for k in range(c_first, c)), (v, c_first, c, published)
            assert sorted(pieces[v]) == list(range(c_first, c + 1))
            written[v] += 1
    assert (edge_seen == 1).all()
    assert (written == 1).all(), np.nonzero(written != 1)


@pytest.mark.parametrize('seed', range(40))
def test_edge_split_covers_every_edge_and_node_once(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 400))
    deg = rng.integers(0, 60, n)
    deg[rng.random(n) < 0.2] = 0                     # empty nodes
    if seed % 5 == 0:
        deg[rng.integers(0, n)] = 5000               # one node spanning many CTAs
    rowptr = np.concatenate([[0], np.cumsum(deg)])
    E = int(rowptr[-1])
    for G in (1, 2, 3, 148, 296):
        if E >= 2 * G:
            simulate(rowptr, G)


def test_single_node_graph():
    simulate(np.array([0, 1000]), 148)
    simulate(np.array([0, 0, 1000, 1000]), 148)
