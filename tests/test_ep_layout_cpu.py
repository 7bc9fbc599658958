"""CPU check of the peer-memory exchange layout that ep_counts_kernel builds
(localai_b200/csrc/ep.cu, ep_counts_kernel), restated here in Python.

Every rank knows the routed-row counts cnt[s][v] of every source rank s and
virtual expert v = owner * E_loc + local.  Rank ``me`` derives:
  run_off[e * G + s]  first receive row of the rows source s sends for my local
                      expert e (receive buffer expert-major, source-minor);
  grp_off[e]          first receive row of local expert e (one GEMM group);
  ret_base[e * G + s] first slot of that run in source s's slot order (where
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
    """The arithmetic of ep_counts_kernel for rank ``me`` (cnt: [G, G * El])."""
    E = G * El
    vme = me * El
    run_off = np.zeros(E + 1, np.int64)
    ret_base = np.zeros(E, np.int64)
    dst_off = np.zeros(E, np.int64)
    grp_off = np.zeros(El + 1, np.int64)
    for i in range(E):
        e, s = i // G, i % G
        r = sum(cnt[s2][vme + e2] for e2 in range(e) for s2 in range(G)) + sum(cnt[s2][vme + e] for s2 in range(s))
        run_off[i] = r
        ret_base[i] = sum(cnt[s][v] for v in range(vme + e))
        d, e2 = i // El, i % El
        dst_off[i] = (sum(cnt[s2][d * El + e3] for e3 in range(e2) for s2 in range(G))
                      + sum(cnt[s2][i] for s2 in range(me)))
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
        # receive runs tile [0, total) in (expert, source) order
        sizes = np.array([cnt[i % G][me * El + i // G] for i in range(E)])
        assert np.array_equal(run_off[1:E] - run_off[:E - 1], sizes[:-1])
        assert run_off[E] == sizes.sum() == grp_off[El]
        assert np.array_equal(grp_off[:El], run_off[0:E:G])
        # what every source writes for my expert e lands on my run (e, source)
        for s in range(G):
            for e in range(El):
                assert lays[s][3][me * El + e] == run_off[e * G + s]
                # outputs go back to the source's slots of virtual expert me*El+e
                assert ret_base[e * G + s] == cnt[s][:me * El + e].sum()
        # the receive buffer holds exactly the rows the NCCL transport would deliver
        send, recv = nccl_splits(cnt, me, G, El)
        assert sum(recv) == run_off[E]
        for d in range(G):
            assert send[d] == cnt[me][d * El:(d + 1) * El].sum()
            assert lays[d][0][E] == sum(int(cnt[s][d * El:(d + 1) * El].sum()) for s in range(G))
