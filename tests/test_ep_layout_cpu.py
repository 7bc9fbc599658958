"""CPU check of the peer-memory exchange layout that ep_counts_kernel builds
(localai_b200/csrc/ep.cu, ep_counts_kernel), restated here in Python.

Every rank knows the routed-row counts cnt[s][v] of every source rank s and
virtual expert v = owner * E_loc + local.  Rank ``me`` derives:
  run_off[e * G + j]  first receive row of the rows source (me + j) % G sends
                      for my local expert e (receive buffer expert-major; in
                      a group my own rows first, then ranks me+1, ...);
  grp_off[e]          first receive row of local expert e (one GEMM group);
  ret_base[e * G + j] first slot of that run in its source's slot order (where
                      the down GEMM writes the outputs back);
  dst_off[d * E_loc + e]  first row in rank d's receive buffer of the rows I
                      send for d's local expert e.
The checks: what a sender writes is exactly where the receiver expects it,
runs tile the receive buffer without gaps or overlaps, outputs land on the
sender's own slots, and the per-(source, expert) row counts equal the split
sizes the NCCL all-to-all transport exchanges.
"""
import numpy as np
import pytest


def layout(cnt, me, G, El):
    """The arithmetic of ep_counts_kernel for rank ``me`` (cnt: [G, G * El]).
    Runs of a receive group are in the source order me, me+1, ...: run j of
    group e comes from source (me + j) % G."""
    E = G * El
    vme = me * El
    run_off = np.zeros(E + 1, np.int64)
    ret_base = np.zeros(E, np.int64)
    dst_off = np.zeros(E, np.int64)
    grp_off = np.zeros(El + 1, np.int64)
    for i in range(E):
        e, j = i // G, i % G
        s = (me + j) % G
        r = (sum(cnt[s2][vme + e2] for e2 in range(e) for s2 in range(G))
             + sum(cnt[(me + j2) % G][vme + e] for j2 in range(j)))
        run_off[i] = r
        ret_base[i] = sum(cnt[s][v] for v in range(vme + e))
        d, e2 = i // El, i % El
        dst_off[i] = (sum(cnt[s2][d * El + e3] for e3 in range(e2) for s2 in range(G))
                      + sum(cnt[(d + j2) % G][i] for j2 in range((me - d) % G)))
    for e in range(El + 1):
        grp_off[e] = sum(cnt[s2][vme + e2] for e2 in range(e) for s2 in range(G))
    run_off[E] = grp_off[El]
    return run_off, grp_off, ret_base, dst_off


def nccl_splits(cnt, me, G, El):
    """Rows rank ``me`` sends to / receives from each rank on the NCCL path
    (localai_b200/ep.py EPMoE.forward): per-destination sums of its own
    counts, and per-source sums of the counts addressed to its experts."""
    send = [int(cnt[me][d * El:(d + 1) * El].sum()) for d in range(G)]
    recv = [int(cnt[s][me * El:(me + 1) * El].sum()) for s in range(G)]
    return send, recv


@pytest.mark.parametrize('G,El,seed', [(1, 4, 0), (2, 8, 1), (4, 16, 2), (8, 8, 3), (8, 32, 4)])
def test_p2p_layout_is_consistent(G, El, seed):
    rng = np.random.default_rng(seed)
    E = G * El
    # skewed counts with zeros, as a Zipf router produces
    cnt = rng.poisson(lam=rng.pareto(1.1, size=E) * 40, size=(G, E)).astype(np.int64)
    cnt[:, rng.choice(E, size=E // 4, replace=False)] = 0
    lays = [layout(cnt, me, G, El) for me in range(G)]
    for me in range(G):
        run_off, grp_off, ret_base, dst_off = lays[me]
        # receive runs tile [0, total) in (expert, source me + j) order
        sizes = np.array([cnt[(me + i % G) % G][me * El + i // G] for i in range(E)])
        assert np.array_equal(run_off[1:E] - run_off[:E - 1], sizes[:-1])
        assert run_off[E] == sizes.sum() == grp_off[El]
        assert np.array_equal(grp_off[:El], run_off[0:E:G])
        # what every source writes for my expert e lands on my run (e, (s - me) mod G)
        for s in range(G):
            j = (s - me) % G
            for e in range(El):
                assert lays[s][3][me * El + e] == run_off[e * G + j]
                # outputs go back to the source's slots of virtual expert me*El+e
                assert ret_base[e * G + j] == cnt[s][:me * El + e].sum()
        # the receive buffer holds exactly the rows the NCCL transport would deliver
        send, recv = nccl_splits(cnt, me, G, El)
        assert sum(recv) == run_off[E]
        for d in range(G):
            assert send[d] == cnt[me][d * El:(d + 1) * El].sum()
            assert lays[d][0][E] == sum(int(cnt[s][d * El:(d + 1) * El].sum()) for s in range(G))


def rounds_tables(cnt, G, El, tile=256, target=16, first=8):
    """Every rank's group row offsets and row-tile bases, and the round
    sizes, as ep_counts_kernel computes them for the fused exchange."""
    dgrp = np.zeros((G, El + 1), np.int64)
    dtile = np.zeros((G, El + 1), np.int64)
    for d in range(G):
        for g in range(El):
            m = int(cnt[:, d * El + g].sum())
            dgrp[d, g + 1] = dgrp[d, g] + m
            dtile[d, g + 1] = dtile[d, g] + (m + tile - 1) // tile
    qmax = int(dtile[:, El].max())
    rt = max(1, (qmax + target - 1) // target)
    r0 = min(rt, first)
    rounds = 0 if qmax == 0 else 1 if qmax <= r0 else 1 + (qmax - r0 + rt - 1) // rt
    return dgrp, dtile, r0, rt, rounds


def round_first_tile(r, r0, rt):
    return 0 if r == 0 else r0 + (r - 1) * rt


def push_plan(cnt, me, G, El, NW, tile=256):
    """(round, warp, d, row) of every row source ``me`` stores, following
    ep_push_rows (localai_b200/csrc/gemm_tc.cu)."""
    dgrp, dtile, r0, rt, rounds = rounds_tables(cnt, G, El, tile)
    _, _, _, dst_off = layout(cnt, me, G, El)
    out = []
    for r in range(rounds):
        q0, q1 = round_first_tile(r, r0, rt), round_first_tile(r + 1, r0, rt)
        acc = 0
        for dd in range(1, G + 1):
            d = (me + dd) % G
            for g in range(El):
                t0, t1 = dtile[d, g], dtile[d, g + 1]
                if t1 <= q0 or t0 >= q1:
                    continue
                row0 = dgrp[d, g] + tile * max(q0 - t0, 0)
                row1 = min(dgrp[d, g] + tile * (q1 - t0), dgrp[d, g + 1])
                v = d * El + g
                base, nv = dst_off[v], cnt[me, v]
                lo, hi = max(row0, base), min(row1, base + nv)
                if hi <= lo:
                    continue
                for w in range(NW):
                    first = lo + (w - acc) % NW
                    for row in range(first, hi, NW):
                        out.append((r, w, d, row))
                acc += hi - lo
    return out, dgrp, dtile, (r0, rt), rounds


@pytest.mark.parametrize('G,El,seed,scale', [(2, 32, 5, 40), (4, 16, 6, 40), (8, 8, 7, 40), (8, 8, 8, 400),
                                              (2, 4, 9, 3)])
def test_fused_exchange_rounds_cover_every_row_once(G, El, seed, scale):
    """The fused exchange's push plan: every row of every receiver is stored
    exactly once, by its own source, in the round of the GEMM row tile that
    holds it; the warps' shares of a round differ by at most one row per
    segment; at most 18 rounds."""
    rng = np.random.default_rng(seed)
    E = G * El
    cnt = rng.poisson(lam=rng.pareto(1.1, size=E) * scale, size=(G, E)).astype(np.int64)
    cnt[:, rng.choice(E, size=E // 4, replace=False)] = 0
    NW = 148
    lays = [layout(cnt, me, G, El) for me in range(G)]
    seen = {d: {} for d in range(G)}
    for me in range(G):
        plan, dgrp, dtile, (r0, rt), rounds = push_plan(cnt, me, G, El, NW)
        assert rounds <= 18
        for r, w, d, row in plan:
            assert row not in seen[d], (d, row)
            seen[d][row] = (me, r)
    for d in range(G):
        run_off, grp_off, _, _ = lays[d]
        total = int(run_off[G * El])
        assert sorted(seen[d]) == list(range(total))
        for row, (s, r) in seen[d].items():
            g = int(np.searchsorted(grp_off[1:El + 1], row, side='right'))
            assert grp_off[g] <= row < grp_off[g + 1]
            e_j = g * G + (s - d) % G                        # the run of source s in group g holds the row
            assert run_off[e_j] <= row < run_off[e_j + 1]
            q = dtile[d, g] + (row - grp_off[g]) // 256      # its GEMM row tile
            assert (0 if q < r0 else 1 + (q - r0) // rt) == r
