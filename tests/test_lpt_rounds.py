"""The plan kernel's parallel LPT (equal-weight runs handed out round by round) equals the
reference's one-task-at-a-time LPT.  A pure-Python model of the kernel's algorithm
(sgld_plan.cu, static_lists_parallel) is compared with the oracle on random cases."""
import random

import pytest

from oracle import planning as P


def rounds_lpt(weights, groups, workers):
    """Model of the kernel: runs of equal weight, rounds (q_i, rho_i), rank by (rho, i)."""
    order = sorted(range(len(weights)), key=lambda i: (-weights[i], i))
    loads = [0] * workers
    heads, links, tails = [-1] * workers, {}, [-1] * workers
    i = 0
    while i < len(order):
        j = i
        while j < len(order) and weights[order[j]] == weights[order[i]]:
            j += 1
        w, run = weights[order[i]], order[i:j]
        k = len(run) * groups
        v0 = min(loads)
        q = [(l - v0) // w for l in loads]
        rho = [(l - v0) % w for l in loads]
        ranked = sorted(range(workers), key=lambda x: (rho[x], x))
        assigned = [[] for _ in range(workers)]
        c, rnd = 0, 0
        while rnd < max(q) and c < k:
            part = [x for x in ranked if q[x] <= rnd]
            for pos, x in enumerate(part):
                if c + pos < k:
                    assigned[x].append(c + pos)
            c += len(part)
            rnd += 1
        for rank, x in enumerate(ranked):
            assigned[x] += list(range(c + rank, k, workers))
        for x in range(workers):
            for jj in sorted(assigned[x]):
                task = run[jj // groups] * groups + jj % groups
                if tails[x] < 0:
                    heads[x] = task
                else:
                    links[tails[x]] = task
                links[task] = -1
                tails[x] = task
            loads[x] += len(assigned[x]) * w
        i = j
    return heads, links


@pytest.mark.parametrize("seed", range(300))
def test_round_lpt_equals_reference_lpt(seed):
    rng = random.Random(seed)
    n = rng.randint(0, 300)
    wmax = rng.choice([1, 2, 4, 16, 64, 1024])
    weights = [rng.randint(1, wmax) for _ in range(n)]
    if rng.random() < 0.3:
        weights = [rng.choice([1, wmax]) for _ in range(n)]
    groups = rng.choice([1, 2, 4, 7, 8])
    workers = rng.choice([1, 2, 3, 5, 37, 148])
    g = P.Geometry(4096, 1, 1, groups, workers)
    want = P._greedy_lists(weights, n, g)
    got = rounds_lpt(weights, groups, workers)
    assert got[0] == want[0]
    assert got[1] == want[1]
