"""CPU model of the expert-parallel combine over peer memory
(exchange_combine_kernel, pokitlms_b200/csrc/pokit_grouped.cu).

Each rank's call c (c = 1, 2, ...) takes the kernel's three steps:
  1. store its partial into slot [c & 1][rank] of every rank's region;
  2. raise flag [c & 1][rank] = c on every rank (after its stores);
  3. wait until flag [c & 1][src] == c for every src of its own region, then
     read slots [c & 1][0..N) and add them in rank order.
The model runs N ranks under random interleavings of these atomic steps and
checks what the kernel relies on: every rank sums exactly the N partials of
the same call (a rank that runs ahead never overwrites a slot another rank
has yet to read), the sums agree across ranks, and a rank that stops before
raising its flag makes the others' bounded waits run out instead of reading
stale data.
"""
import random


def run(n_ranks, calls, seed, stop_rank=None, stop_call=None, spin_limit=10_000):
    rng = random.Random(seed)
    slots = [[[None] * n_ranks for _ in range(2)] for _ in range(n_ranks)]   # [owner][parity][src]
    flags = [[[0] * n_ranks for _ in range(2)] for _ in range(n_ranks)]
    # rank state: (call, phase), phase 0 = store, 1 = flag, 2 = wait/read
    state = [[1, 0, 0] for _ in range(n_ranks)]   # call, phase, spins
    results = [[] for _ in range(n_ranks)]
    timeouts = [0] * n_ranks

    def partial(rank, call):
        return (rank + 1) * 1000 + call

    active = set(range(n_ranks))
    while active:
        r = rng.choice(sorted(active))
        call, phase, spins = state[r]
        par = call & 1
        if phase == 0:
            if stop_rank == r and stop_call == call:
                active.discard(r)          # this rank never stores or raises its flag
                continue
            for d in range(n_ranks):
                slots[d][par][r] = (call, partial(r, call))
            state[r] = [call, 1, 0]
        elif phase == 1:
            for d in range(n_ranks):
                flags[d][par][r] = call
            state[r] = [call, 2, 0]
        else:
            if all(flags[r][par][s] == call for s in range(n_ranks)):
                got = [slots[r][par][s] for s in range(n_ranks)]
                assert all(g[0] == call for g in got), (r, call, got)
                results[r].append(sum(g[1] for g in got))
                nxt = call + 1
                if nxt > calls:
                    active.discard(r)
                state[r] = [nxt, 0, 0]
            elif spins + 1 > spin_limit:
                timeouts[r] += 1
                active.discard(r)          # the kernel sets the status bit; the host stops
            else:
                state[r] = [call, 2, spins + 1]
    return results, timeouts


def test_every_rank_sums_the_same_call_under_any_interleaving():
    for n in (2, 3, 4, 8):
        for seed in range(40):
            results, timeouts = run(n, calls=12, seed=seed)
            assert timeouts == [0] * n
            want = [sum((r + 1) * 1000 + c for r in range(n)) for c in range(1, 13)]
            for r in range(n):
                assert results[r] == want


def test_a_rank_that_stops_makes_the_others_time_out_not_read_stale_slots():
    for n in (2, 4, 8):
        for seed in range(20):
            results, timeouts = run(n, calls=6, seed=seed, stop_rank=n - 1, stop_call=4, spin_limit=200)
            for r in range(n - 1):
                assert len(results[r]) == 3        # calls 1..3 complete, call 4 never does
                assert timeouts[r] == 1


def exchange_bytes(world, max_tokens, hidden):
    """ep_exchange_bytes: partials [2][world][max_tokens][hidden] F32, then
    [2][world] uint32 flags, rounded up to 256 bytes."""
    b = 2 * world * max_tokens * hidden * 4 + 2 * world * 4
    return (b + 255) // 256 * 256


def test_exchange_offsets_stay_inside_the_region():
    """The byte offsets exchange_combine_kernel forms: float4 partial stores
    and loads at ((par * world + src) * slot + t * hidden + 4c) * 4, flags at
    2 * world * slot * 4 + (par * world + src) * 4."""
    for world in (1, 2, 3, 4, 8):
        for max_tokens in (1, 7, 16, 64):
            for hidden in (256, 2048, 4096):
                region = exchange_bytes(world, max_tokens, hidden)
                slot = max_tokens * hidden
                last_float4 = ((1 * world + (world - 1)) * slot + (max_tokens - 1) * hidden + hidden - 4) * 4
                assert last_float4 + 16 <= 2 * world * slot * 4           # partials end before the flags
                flags0 = 2 * world * slot * 4
                last_flag = flags0 + (1 * world + (world - 1)) * 4
                assert last_flag + 4 <= region
                assert flags0 % 4 == 0 and (slot * 4) % 16 == 0         # aligned flags and float4 slots
