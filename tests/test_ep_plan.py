"""Host arithmetic of the peer-copy EP exchange (moe_b200.ep.exchange_plan).

Simulates every rank's copies into the peers' receive and return buffers with
the plan's offsets and checks them against the all-to-all semantics: rank d's
receive buffer holds the blocks of ranks 0..G-1 in order, each block in the
sender's expert-major order, and the combine puts every row back where its
sender's permuted buffer had it.
"""
import numpy as np
import pytest

from moe_b200.ep import ep_group_table, exchange_plan, expert_major_layout, pull_group_table


@pytest.mark.parametrize("world,experts", [(2, 8), (4, 16), (8, 256)])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_exchange_plan_matches_all_to_all(world, experts, seed):
    rng = np.random.default_rng(seed + world)
    el = experts // world
    counts = rng.integers(0, 50, size=(world, experts))
    counts[rng.random(counts.shape) < 0.3] = 0
    plans = [exchange_plan(counts.tolist(), r, el) for r in range(world)]
    # each rank's permuted rows, labelled (source rank, local row index)
    xp = [np.stack([np.full(counts[r].sum(), r), np.arange(counts[r].sum())], 1) for r in range(world)]
    recv = [np.full((world * counts.sum(), 2), -1) for _ in range(world)]
    for r, p in enumerate(plans):
        for d in range(world):
            rows = xp[r][p.send_off[d]:p.send_off[d] + p.send[d]]
            recv[d][p.dst_off[d]:p.dst_off[d] + p.send[d]] = rows
    for d, p in enumerate(plans):
        # all-to-all layout: source blocks in rank order
        expect = np.concatenate([xp[s][plans[s].send_off[d]:plans[s].send_off[d] + plans[s].send[d]]
                                 for s in range(world)])
        got = recv[d][:sum(p.recv)]
        np.testing.assert_array_equal(got, expect)
        assert p.recv_off == list(np.concatenate([[0], np.cumsum(p.recv)[:-1]]))
        # the (source, local expert) segments the grouped GEMM walks
        rc = counts[:, d * el:(d + 1) * el].reshape(-1)
        starts, rows, widx = ep_group_table(rc.tolist(), world, el)
        assert sum(rows) == sum(p.recv)
        for g, (st, n, w) in enumerate(zip(starts, rows, widx)):
            src = g % world
            assert np.all(got[st:st + n, 0] == src)
    # combine: results travel back with back_off and must land at the sender's rows
    ret = [np.full((counts[r].sum(), 2), -1) for r in range(world)]
    for d, p in enumerate(plans):
        got = recv[d][:sum(p.recv)]
        for s in range(world):
            blk = got[p.recv_off[s]:p.recv_off[s] + p.recv[s]]
            ret[s][p.back_off[s]:p.back_off[s] + p.recv[s]] = blk
    for r in range(world):
        np.testing.assert_array_equal(ret[r], xp[r])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_balanced_placement(world):
    from moe_b200.ep import balanced_placement
    rng = np.random.default_rng(world)
    e = 256
    load = (rng.pareto(1.5, e) * 100).astype(int)
    pl = balanced_placement(load.tolist(), world)
    assert sorted(pl) == list(range(e))
    per = e // world
    tot = [sum(load[pl[r * per:(r + 1) * per]]) for r in range(world)]
    contig = [sum(load[r * per:(r + 1) * per]) for r in range(world)]
    assert max(tot) <= max(contig)
    # LPT bound: the heaviest rank exceeds the mean by at most the largest single expert
    assert max(tot) - np.mean(tot) <= load.max() + 1e-9
    for r in range(world):
        assert pl[r * per:(r + 1) * per] == sorted(pl[r * per:(r + 1) * per])


@pytest.mark.parametrize("world,experts", [(1, 8), (2, 8), (4, 16), (8, 256)])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_expert_major_layout(world, experts, seed):
    """Fused-transport layout: every sender's row of expert e lands at its
    permuted row + deltas[e] in the owner's buffer; the owner's buffer holds
    its local experts in order, each as one block of sources 0..G-1 in order,
    with nothing overlapping and nothing left empty."""
    rng = np.random.default_rng(seed + 10 * world)
    el = experts // world
    counts = rng.integers(0, 60, size=(world, experts))
    counts[rng.random(counts.shape) < 0.3] = 0
    lays = [expert_major_layout(counts.tolist(), r, el) for r in range(world)]
    tot = counts.sum(0)
    recv = [np.full((world * counts.sum(), 3), -1) for _ in range(world)]
    for s, lay in enumerate(lays):
        start = np.concatenate([[0], np.cumsum(counts[s])[:-1]])
        for e in range(experts):
            d = e // el
            for i in range(counts[s, e]):
                row = start[e] + i + lay.deltas[e]
                assert 0 <= row < lay.recv_rows[d]
                assert recv[d][row, 0] == -1, "two rows land on one slot"
                recv[d][row] = (e, s, i)
    for d in range(world):
        lay = lays[d]
        assert lay.splits == list(tot[d * el:(d + 1) * el])
        assert lay.recv_rows == [int(tot[q * el:(q + 1) * el].sum()) for q in range(world)]
        expect = [(d * el + j, s, i) for j in range(el) for s in range(world)
                  for i in range(counts[s, d * el + j])]
        np.testing.assert_array_equal(recv[d][:lay.recv_rows[d]], np.array(expect).reshape(-1, 3))
        assert (recv[d][lay.recv_rows[d]:] == -1).all()


@pytest.mark.parametrize("el,chunks", [(32, 2), (32, 3), (2, 2), (7, 4), (128, 1)])
def test_overlap_chunks_cover_every_local_expert_once(el, chunks):
    """The overlapped EP path dispatches and multiplies the local experts in
    contiguous chunks; together they must cover each local expert once, in
    order (so the receive rows and GEMM groups equal the unchunked ones)."""
    from moe_b200.ep import MoELayerEP
    bounds = MoELayerEP.chunk_bounds(el, chunks)
    assert len(bounds) == chunks
    assert bounds[0][0] == 0 and bounds[-1][1] == el
    for (a, b), (c, d) in zip(bounds, bounds[1:]):
        assert a < b and b == c
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world,experts", [(2, 8), (4, 16), (8, 256)])
@pytest.mark.parametrize("seed", [0, 1])
def test_pull_group_table_matches_push_layout(world, experts, seed):
    """The pull dispatch's group table sends every receive row to the source
    permuted row that the push dispatch stores there (row + deltas_s[e])."""
    rng = np.random.default_rng(seed)
    counts = rng.integers(0, 40, size=(world, experts))
    counts[:, rng.integers(0, experts, 3)] = 0  # some empty (source, expert) blocks
    el = experts // world
    for rank in range(world):
        lay = expert_major_layout(counts.tolist(), rank, el)
        n = sum(lay.splits)
        push = np.full(n, -1)
        pull = np.full(n, -1)
        for s in range(world):
            deltas = expert_major_layout(counts.tolist(), s, el).deltas
            src_start = np.cumsum(counts[s]) - counts[s]
            for le in range(el):
                e = rank * el + le
                for j in range(counts[s, e]):
                    push[src_start[e] + j + deltas[e]] = s * 1000000 + src_start[e] + j
        start, cnt, src0 = pull_group_table(counts.tolist(), rank, el)
        assert start == sorted(start) and start[0] == 0
        for g, (a, c, r0) in enumerate(zip(start, cnt, src0)):
            s = g % world
            for j in range(c):
                pull[a + j] = s * 1000000 + r0 + j
        assert np.array_equal(push, pull) and (pull >= 0).all()
