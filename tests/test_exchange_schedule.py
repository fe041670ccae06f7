"""The fused row-parallel exchange cannot deadlock: a host-side simulation of its schedule.

gemv_tc.cu splits a rank's units (128-row group x 256-column stage) over its CTAs as
u0 = b * U / grid (stream-K), and a CTA's epilogue finishes its segments in order. The CTA whose
contribution completes a row group pushes the group's rows to every rank and then waits until
every rank has pushed that group before it moves on. Ranks may split K differently (TP 8 cuts
down_proj into 1792- and 2048-column shards), so their unit partitions differ. This simulation
runs every CTA of every rank as a sequential process under random interleavings and checks that
all of them finish. That is the no-deadlock argument in the kernel's comment, exercised on the
shapes the 12B-class model uses at TP 2, 4 and 8 and on random ones.
"""
import random

import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402


def _segments(u0, u1, n_stages):
    """(row group, number of units) per segment of the unit range [u0, u1), in order."""
    out, u = [], u0
    while u < u1:
        rg = u // n_stages
        end = min(u1, (rg + 1) * n_stages)
        out.append((rg, end - u))
        u = end
    return out


def simulate(row_groups, stages_per_rank, sms, seed, reversed_ranks=()):
    """True if every CTA of every rank finishes under a random interleaving. The CTAs of
    ``reversed_ranks`` take their segments in reverse order (not what the kernel does: the
    control case that must be able to deadlock)."""
    rng = random.Random(seed)
    world = len(stages_per_rank)
    ctas = []                                    # (rank, list of segments)
    for r, ns in enumerate(stages_per_rank):
        U = row_groups * ns
        grid = min(sms, U)
        for b in range(grid):
            segs = _segments(b * U // grid, (b + 1) * U // grid, ns)
            ctas.append((r, segs[::-1] if r in reversed_ranks else segs))
    done_units = [[0] * row_groups for _ in range(world)]
    pushed = [[False] * row_groups for _ in range(world)]
    pos = [0] * len(ctas)                        # next segment of each CTA
    waiting = [None] * len(ctas)                 # row group a finaliser waits on
    live = set(range(len(ctas)))
    while live:
        runnable = []
        for c in live:
            rg = waiting[c]
            if rg is None or all(pushed[q][rg] for q in range(world)):
                runnable.append(c)
        if not runnable:
            return False
        c = rng.choice(runnable)
        r, segs = ctas[c]
        if waiting[c] is not None:               # the exchange of this group completed
            waiting[c] = None
            pos[c] += 1
        else:
            rg, units = segs[pos[c]]
            done_units[r][rg] += units
            if done_units[r][rg] == stages_per_rank[r]:
                pushed[r][rg] = True             # this CTA finalises the group on rank r
                waiting[c] = rg
            else:
                pos[c] += 1
        if waiting[c] is None and pos[c] == len(segs):
            live.discard(c)
    return all(all(p) for p in pushed)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("k", [4096, 15360])            # o_proj, down_proj of the 12B-class model
def test_model_shapes_finish(world, k):
    from flashbfp_b200 import tp
    stages = []
    for r in range(world):
        lo, hi = tp.split(k, r, world, align=tp.ROW_K_ALIGN)
        stages.append((hi - lo) // 256)
    for seed in range(20):
        assert simulate(3840 // 128, stages, 148, seed), (world, k, stages, seed)


@settings(max_examples=150, deadline=None)
@given(world=st.sampled_from([2, 3, 4, 8]), row_groups=st.integers(1, 12),
       stages=st.lists(st.integers(1, 24), min_size=8, max_size=8), sms=st.integers(1, 40),
       seed=st.integers(0, 10_000))
def test_random_shapes_finish(world, row_groups, stages, sms, seed):
    assert simulate(row_groups, stages[:world], sms, seed)


def test_out_of_order_finishing_is_caught():
    """The simulation detects a deadlock: with one CTA per rank covering two row groups, a rank
    that finishes group 1 first waits for the other rank's push of group 1, which that rank
    makes only after its own group 0 exchange, which needs the first rank's group 0."""
    assert simulate(2, [4, 4], 1, 0)
    assert not simulate(2, [4, 4], 1, 0, reversed_ranks=(0,))
