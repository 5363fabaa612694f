"""The peer-memory exchange plan (the arithmetic plan_kernel runs on the
device, exported as noor_moe_peer_plan) for 2, 4 and 8 ranks, on the CPU:
every rank's picks of every expert land exactly in the owner's receive group
for (expert, sender), the groups tile each owner's receive buffer, and every
output row goes back to the sender's own pick row."""
import numpy as np
import pytest


def _plans(pkg, cnt, BM):
    return [pkg.api.peer_plan(cnt, me, BM) for me in range(cnt.shape[0])]


@pytest.mark.parametrize("G,E", [(2, 32), (4, 32), (8, 32), (8, 64), (4, 8), (8, 128)])
@pytest.mark.parametrize("pattern", ["uniform", "ragged", "empty_rank", "one_hot"])
def test_plan_routes_every_pick_home(pkg, G, E, pattern):
    rng = np.random.default_rng(G * 1000 + E)
    if pattern == "uniform":
        cnt = rng.integers(100, 600, size=(G, E))
    elif pattern == "ragged":
        cnt = rng.integers(0, 900, size=(G, E)) * (rng.random((G, E)) < 0.7)
    elif pattern == "empty_rank":
        cnt = rng.integers(0, 400, size=(G, E))
        cnt[G // 2] = 0
    else:
        cnt = np.zeros((G, E), np.int64)
        cnt[:, E - 1] = rng.integers(1, 5000, size=G)  # every token on the last rank's last expert
    cnt = cnt.astype(np.int64)
    El, BM = E // G, 256
    plans = _plans(pkg, cnt, BM)
    pre = np.concatenate([np.zeros((G, 1), np.int64), np.cumsum(cnt, axis=1)], axis=1)  # source layouts
    for r, p in enumerate(plans):
        assert np.array_equal(p["counts_glob"], cnt.sum(axis=0))
        # the groups tile [0, total) in order; tiles count whole BM-row tiles per group
        rows = np.diff(p["grp_row"])
        assert p["grp_row"][0] == 0 and (rows >= 0).all()
        assert p["grp_row"][-1] == cnt[:, r * El:(r + 1) * El].sum()
        assert np.array_equal(np.diff(p["grp_mtile"]), (rows + BM - 1) // BM)
        for j in range(E):
            le, src = divmod(j, G)
            e = r * El + le
            assert p["grp_widx"][j] == le and p["grp_orank"][j] == src
            assert rows[j] == cnt[src, e]
            # the sender stores its picks of e at dest_base and gets them back at its own rows
            assert plans[src]["dest_base"][e] == p["grp_row"][j]
            assert p["grp_row"][j] + p["grp_oshift"][j] == pre[src, e]


def test_plan_rejects_bad_arguments(pkg):
    with pytest.raises(pkg.api.NoorMoEError):
        pkg.api.peer_plan(np.zeros((3, 8), np.int64), 0, 256)  # E not divisible by G
    with pytest.raises(pkg.api.NoorMoEError):
        pkg.api.peer_plan(np.full((2, 8), -1, np.int64), 0, 256)
    with pytest.raises(pkg.api.NoorMoEError):
        pkg.api.peer_plan(np.zeros((9, 9), np.int64), 0, 256)  # more ranks than the exchange supports
