"""The plan kernel's parallel LPT (equal-weight runs handed out round by round) equals the
reference's one-task-at-a-time LPT.  A pure-Python model of the kernel's algorithm
(sgld_plan.cu, static_lists_runs) is compared with the oracle on random cases."""
import random

import pytest

from oracle import planning as P


def rounds_lpt(weights, groups, workers):
    """Model of the kernel (sgld_plan.cu, static_lists_runs), step for step.

    Runs come heaviest first; (q, rho) are taken against a zero baseline, rounds run from
    min q to max q - 1; the
    thread of rank t acts for worker rank_of[t]; pre-steady rounds hand out (round, rho, i)
    slots; steady rounds give rank t tasks c + t + m*W with next[task(j)] = task(j + W)
    written task-parallel; a worker's last task gets -1 at the end.  Every next[] entry
    must be written exactly once (the kernel relies on it)."""
    n = len(weights)
    loads, tails, heads = [0] * workers, [-1] * workers, [-1] * workers
    links, writes = {}, {}

    def write(task, value):
        writes[task] = writes.get(task, 0) + 1
        links[task] = value

    prev_w, consumed = 2**31 - 1, 0
    while consumed < n:
        w = max(x for x in weights if x < prev_w)
        v0 = 0                                                   # any lower bound of the loads
        run = [i for i in range(n) if weights[i] == w]           # ascending record ids
        k = len(run) * groups
        q = [(l - v0) // w for l in loads]
        rho = [(l - v0) % w for l in loads]
        rank_of = sorted(range(workers), key=lambda x: (rho[x], x))
        task_of = lambda j: run[j // groups] * groups + j % groups
        state = {}
        for t, at in enumerate(rank_of):
            state[t] = [at, q[at], tails[at], heads[at], 0]          # at, q, tail, head, assigned

        def take(t, j):
            st = state[t]
            task = task_of(j)
            if st[2] < 0:
                st[3] = task
            else:
                write(st[2], task)
            st[2] = task
            st[4] += 1

        c, rnd = 0, min(q)
        while rnd < max(q) and c < k:
            part = [t for t in range(workers) if state[t][1] <= rnd]   # thread order = rank order
            for pos, t in enumerate(part):
                if c + pos < k:
                    take(t, c + pos)
            c += len(part)
            rnd += 1
        for t in range(workers):
            if c + t < k:
                j0 = c + t
                m = (k - 1 - j0) // workers
                take(t, j0)
                state[t][2] = task_of(j0 + m * workers)
                state[t][4] += m
        for j in range(c, k):
            if j + workers < k:
                write(task_of(j), task_of(j + workers))
        for t in range(workers):
            at, _, tail, head, assigned = state[t]
            loads[at] += assigned * w
            tails[at], heads[at] = tail, head
        consumed += len(run)
        prev_w = w
    for x in range(workers):
        if tails[x] >= 0:
            write(tails[x], -1)
    assert all(v == 1 for v in writes.values()), "a next[] entry was written twice"
    assert len(writes) == n * groups, "a task has no next[] entry"
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
