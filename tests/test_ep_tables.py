"""CPU check of the offset tables the NVLink exchange builds on the device
(csrc/ep_peer.cu, ep_counts_kernel), restated in numpy from the formulas in
that file's header:

  counts[s][g]      rows source rank s routes to global expert g
  cum_s(g)          sum_{g' < g} counts[s][g']       (s's dispatch order is global-expert sorted)
  exp_off_d(e, s)   sum_{e' < e} sum_s' counts[s'][d*El + e'] + sum_{s' < s} counts[s'][d*El + e]
  base_s[g]         exp_off_{g // El}(g % El, s)
  src_pos_d[e, s]   cum_s(d*El + e)

Row p of source s's dispatch order (expert g) is put at base_s[g] + (p - cum_s(g))
of rank g // El's receive region; expert-major row q of rank d in block (e, s)
(j-th of the block) returns to position src_pos_d[e, s] + j of s's return
region.  Over random per-rank counts for 2, 4 and 8 ranks: every receive
region is filled exactly once in (expert, source, arrival) order, which is the
direct all-to-all permutation, and every row returns to the slot it left."""

import numpy as np
import pytest


def tables(counts: np.ndarray, rank: int):
  """The four tables rank `rank` builds, as the device kernel defines them."""
  W, E = counts.shape
  El = E // W
  cum = np.concatenate([[0], np.cumsum(counts[rank])])  # cum_r(g), E + 1 entries
  tot = counts.sum(0)
  tot_scan = np.concatenate([[0], np.cumsum(tot)])
  before = np.array([counts[:rank, g].sum() for g in range(E)], np.int64)
  base = np.array([tot_scan[g] - tot_scan[(g // El) * El] + before[g] for g in range(E)])
  g0 = rank * El
  exp_off = np.zeros(El * W + 1, np.int64)
  src_pos = np.zeros(El * W, np.int64)
  for e in range(El):
    for s in range(W):
      exp_off[e * W + s] = tot_scan[g0 + e] - tot_scan[g0] + counts[:s, g0 + e].sum()
      src_pos[e * W + s] = counts[s, :g0 + e].sum()
  exp_off[El * W] = tot[g0:g0 + El].sum()
  return base, cum, exp_off, src_pos


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_offset_tables_are_the_all_to_all_permutation(world, seed):
  rng = np.random.default_rng(seed * 10 + world)
  E = 16 * world
  El = E // world
  # skewed counts with empty experts, as the router bias produces
  counts = rng.poisson(rng.gamma(0.5, 6.0, size=(1, E)), size=(world, E)).astype(np.int64)
  counts[:, rng.choice(E, size=E // 4, replace=False)] = 0
  tabs = [tables(counts, r) for r in range(world)]
  # every row is identified by (source, position in the source's dispatch order)
  recv = [np.full(counts[:, d * El:(d + 1) * El].sum(), -1, np.int64) for d in range(world)]
  for s in range(world):
    base, cum, _, _ = tabs[s]
    for g in range(E):
      d = g // El
      for p in range(cum[g], cum[g + 1]):
        pos = base[g] + (p - cum[g])
        assert recv[d][pos] == -1, "two rows put at one receive position"
        recv[d][pos] = s * 10**6 + p
  for d in range(world):
    assert (recv[d] >= 0).all(), "receive region not filled"
    # the direct all-to-all in expert-major order: (local expert, source, arrival)
    direct = []
    for e in range(El):
      g = d * El + e
      for s in range(world):
        cum_s = np.concatenate([[0], np.cumsum(counts[s])])
        direct += [s * 10**6 + p for p in range(cum_s[g], cum_s[g + 1])]
    assert np.array_equal(recv[d], np.array(direct, np.int64))
    # local group sizes = rows per local expert over all sources
    _, _, exp_off, _ = tabs[d]
    gs_local = counts[:, d * El:(d + 1) * El].sum(0)
    assert exp_off[El * world] == gs_local.sum()
  # return: expert-major row q of rank d goes back to its source's slot
  for d in range(world):
    _, _, exp_off, src_pos = tabs[d]
    nb = El * world
    for q in range(exp_off[nb]):
      blk = int(np.searchsorted(exp_off[:nb], q, side="right") - 1)
      s = blk % world
      pos = src_pos[blk] + (q - exp_off[blk])
      assert recv[d][q] == s * 10**6 + pos, "row returns to a different slot"
