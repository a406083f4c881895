"""Split of the 20 neuron slices (the reference's "blocks") over the GPUs of
one box, and the owned block ids of each GPU.

compute_shares restates src/planner.c:56-127: each participant has a
nondecreasing completion-time curve over its share; the optimal time limit is
the smallest curve value at which the shares fitting under it cover all
slices; surplus is then removed one slice at a time from the currently
slowest participant, the first index winning ties (strict '>').
assign restates src/head.c:60-81: shares become disjoint ascending id ranges
in participant order.
"""

SLICES = 20


def compute_shares(times, total=SLICES):
    """times[i][b]: participant i's time at share b (b = 0..capacity); returns shares."""
    n = len(times)
    if not n:
        raise ValueError("no participants")
    cap = [len(t) - 1 for t in times]
    if sum(cap) < total:
        raise ValueError("not enough capacity for %d slices" % total)
    # monotone curves (a noisy sweep point never makes more slices look cheaper)
    mono = []
    for t in times:
        m = [0.0]
        for b in range(1, len(t)):
            m.append(max(m[-1], float(t[b])))
        mono.append(m)
    limit = None
    for j in range(n):
        for b in range(1, cap[j] + 1):
            cand = mono[j][b]
            if limit is not None and cand >= limit:
                continue
            fit = 0
            for i in range(n):
                s = 0
                while s < cap[i] and mono[i][s + 1] <= cand:
                    s += 1
                fit += s
            if fit >= total:
                limit = cand
    shares = []
    for i in range(n):
        s = 0
        while s < cap[i] and mono[i][s + 1] <= limit:
            s += 1
        shares.append(s)
    used = sum(shares)
    while used > total:
        slow = None
        for i in range(n):
            if shares[i] and (slow is None or mono[i][shares[i]] > mono[slow][shares[slow]]):
                slow = i
        shares[slow] -= 1
        used -= 1
    return shares


def equal_shares(n_gpus, total=SLICES):
    """Identical GPUs: cost proportional to the share (1 GPU -> 20, 2 -> 10/10,
    4 -> 5 x 4, 8 -> 2,2,2,2,3,3,3,3)."""
    return compute_shares([[float(b) for b in range(total + 1)] for _ in range(n_gpus)], total)


def assign(shares):
    """Owned slice ids per participant: consecutive ascending ranges."""
    out, start = [], 0
    for s in shares:
        out.append(list(range(start, start + s)))
        start += s
    return out


def owned_blocks(rank, world, total=SLICES):
    return assign(equal_shares(world, total))[rank]
