"""CPU checks of the tensor-core GEMV stack (gemm_q4_0_mma_stack_kernel,
nexusllm_b200/csrc/mma_stack_kernels.cuh; mma_stack_create in nexus_gpu.cu),
restated in Python before any GPU run:

* the host plan: the hop groups (tasks from one hop -- a new input, or an
  `after` task not yet behind a barrier -- to the next), their members' tile
  offsets, x slots, conversions and stream-K CTA counts;
* every group's chunks are covered once by its CTAs' ranges, the raw-copy
  warp's incremental walk names the right member, tile and chunk, the CTAs
  the fix-up counts for a shared tile (sk_owner of its first and last chunk)
  are exactly the CTAs that work on it, so a grow-only arrival counter marks
  exactly one last arrival per tile in every run, and the partial-sum slots
  the fix-up reads are the ones its CTAs wrote;
* the two grid barrier counters, simulated with many random interleavings of
  the CTAs' roles over several runs: no conversion starts before every CTA is
  done with the tasks before its hop, no x tile is copied before every CTA
  published its conversion, and nothing deadlocks;
* the shared-memory budget of the kernel.
"""
import random

import pytest

from tests.test_mma_plan import sk_lo, sk_owner, tc_ctas

ROWS, RAW_K = 128, 256
SMS = 148
SMEM_OPTIN = 232448


def stack_plan(tasks, input_cols, sms=SMS):
    """tasks: (rows, cols, x_source, after).  Mirror of mma_stack_create: the
    hop groups (tasks from one hop to the next, one input) with their members'
    tile offsets, stream-K CTAs, the x slot (0: the stack input, converted at
    its first hop of a run; 1: an earlier task's y, converted at every hop) and
    the "published" barrier that covers it.  Returns (groups, tile0 per task)."""
    groups, tile0, last_hop = [], [], 0
    pubs, in_pub, cur_pub = 0, -1, -1
    for i, (rows, cols, src, after) in enumerate(tasks):
        assert cols % RAW_K == 0
        assert (input_cols if src < 0 else tasks[src][0]) == cols
        hop = i == 0 or src != tasks[i - 1][2] or (after >= 0 and after >= last_hop)
        if hop:
            last_hop = i
            conv = src >= 0 or in_pub < 0
            if conv:
                cur_pub = pubs
                pubs += 1
                if src < 0:
                    in_pub = cur_pub
            groups.append(dict(first=i, count=0, tiles=0, nc=cols // RAW_K, hidx=len(groups), conv=conv,
                               pidx=in_pub if src < 0 else cur_pub, xslot=0 if src < 0 else 1, member_tiles=[]))
        g = groups[-1]
        t = -(-rows // ROWS)
        tile0.append(g["tiles"])
        g["member_tiles"].append(t)
        g["tiles"] += t
        g["count"] += 1
    for g in groups:
        g["total"] = g["tiles"] * g["nc"]
        g["G"] = tc_ctas(sms, g["tiles"], g["nc"])
    stack_plan.pubs = pubs
    return groups, tile0


def decode_tasks(layers, h=4096, kv=1024, f=14336, vocab=128256):
    """The bench's decode step: q, k, v (x = stack input, after the previous
    down), o (x = q), gate, up (x = o), down (x = gate); the LM head."""
    t, last_down = [], -1
    for _ in range(layers):
        b = len(t)
        t += [(h, h, -1, last_down), (kv, h, -1, last_down), (kv, h, -1, last_down), (h, h, b, -1),
              (f, h, b + 3, -1), (f, h, b + 3, -1), (h, f, b + 4, -1)]
        last_down = b + 6
    return t + [(vocab, h, -1, last_down)]


def test_hops_of_a_decode_step():
    groups, tile0 = stack_plan(decode_tasks(3), 4096)
    # q+k+v, o, gate+up, down per layer; the head reads the stack input again
    assert [g["count"] for g in groups] == [3, 1, 2, 1] * 3 + [1]
    assert [g["first"] for g in groups[:5]] == [0, 3, 4, 6, 7]
    assert groups[0]["tiles"] == 32 + 8 + 8 and tile0[:3] == [0, 32, 40] and tile0[4:6] == [0, 112]
    # the stack input is converted once (q of layer 0); o, gate and down convert every layer
    assert [g["conv"] for g in groups[:8]] == [True, True, True, True, False, True, True, True]
    assert stack_plan.pubs == 1 + 3 * 3 and not groups[-1]["conv"]
    assert all(groups[i]["pidx"] == 0 and groups[i]["xslot"] == 0 for i in (0, 4, len(groups) - 1))
    for i, g in enumerate(groups):  # a y-input group's barrier is its own conversion
        if g["xslot"]:
            assert g["conv"] and g["pidx"] == sum(h["conv"] for h in groups[:i + 1]) - 1
    # an `after` on the previous task with the same input forces a hop
    groups, _ = stack_plan([(256, 256, -1, -1), (256, 256, -1, 0)], 256)
    assert len(groups) == 2 and not groups[1]["conv"]


def member_walk(g, lo, hi):
    """The raw-copy warp's incremental walk over a CTA's chunks [lo, hi) of a
    group: (member, member tile, chunk) per chunk."""
    nc, mtiles = g["nc"], g["member_tiles"]
    t0 = lo // nc
    m, acc = 0, 0
    while m + 1 < len(mtiles) and acc + mtiles[m] <= t0:  # mma_member
        acc += mtiles[m]
        m += 1
    local, mt, c = t0 - acc, mtiles[m], lo - t0 * nc
    out = []
    for L in range(lo, hi):
        out.append((m, local, c))
        c += 1
        if c == nc:
            c = 0
            local += 1
            if local == mt and L + 1 < hi:
                m, local, mt = m + 1, 0, mtiles[m + 1]
    return out


@pytest.mark.parametrize("layers", [1, 2])
def test_member_walk_and_stream_k_cover(layers):
    groups, tile0 = stack_plan(decode_tasks(layers), 4096)
    for g in groups:
        total, G, nc = g["total"], g["G"], g["nc"]
        assert 1 <= G <= SMS
        seen = {}
        starts = [sum(g["member_tiles"][:m]) for m in range(g["count"])]
        for b in range(G):
            lo, hi = sk_lo(total, G, b), sk_lo(total, G, b + 1)
            assert hi > lo
            for L, (m, local, c) in zip(range(lo, hi), member_walk(g, lo, hi)):
                tile = L // nc
                assert (m, local, c) == (max(k for k in range(g["count"]) if starts[k] <= tile),
                                         tile - starts[m], L % nc)
                assert 0 <= local < g["member_tiles"][m]
                seen[L] = seen.get(L, 0) + 1
        assert sorted(seen) == list(range(total)) and set(seen.values()) == {1}


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096),
                                       (300, 256), (128, 256), (1, 512), (8192, 28672)])
def test_stream_k_cover_and_fixup_arrivals(rows, cols):
    groups, _ = stack_plan([(rows, cols, -1, -1)], cols)
    p = groups[0]
    total, G, nc = p["total"], p["G"], p["nc"]
    seen = [0] * total
    workers = {}
    for b in range(SMS):
        if b >= G:
            continue
        lo, hi = sk_lo(total, G, b), sk_lo(total, G, b + 1)
        assert hi > lo  # every counted CTA has work
        for L in range(lo, hi):
            seen[L] += 1
            workers.setdefault(L // nc, set()).add(b)
    assert seen == [1] * total
    for tile, ws in workers.items():
        bf, bl = sk_owner(total, G, tile * nc), sk_owner(total, G, (tile + 1) * nc - 1)
        assert ws == set(range(bf, bl + 1)), tile
        n = bl - bf + 1
        if n == 1:
            continue
        # grow-only arrival counter over 5 runs: exactly one last arrival per run
        ctr = 0
        for run in range(5):
            lasts = 0
            for _ in ws:
                lasts += ctr % n == n - 1
                ctr += 1
            assert lasts == 1


@pytest.mark.parametrize("layers", [1, 2])
def test_partial_slots_of_a_group(layers):
    """A CTA's partial sums for a group's shared tiles go to slot 2b (its first
    tile) or 2b + 1 (its last); groups are apart by a grid barrier, so two
    slots a CTA suffice.  The fix-up reads slot 2 bb for every sharing CTA
    after the first, and for the first CTA slot 2 bf + 1 exactly when its
    range started in an earlier tile."""
    groups, _ = stack_plan(decode_tasks(layers), 4096)
    for g in groups:
        total, G, nc = g["total"], g["G"], g["nc"]
        written = {}  # tile -> {cta: slot}
        for b in range(G):
            lo, hi = sk_lo(total, G, b), sk_lo(total, G, b + 1)
            t0, t1 = lo // nc, (hi - 1) // nc
            used = set()
            for tile in range(t0, t1 + 1):
                c0 = lo - tile * nc if tile == t0 else 0
                c1 = hi - tile * nc if tile == t1 else nc
                if c0 == 0 and c1 == nc:
                    continue
                slot = 2 * b + (0 if tile == t0 else 1)
                assert slot not in used
                used.add(slot)
                written.setdefault(tile, {})[b] = slot
        for tile, w in written.items():
            bf, bl = sk_owner(total, G, tile * nc), sk_owner(total, G, (tile + 1) * nc - 1)
            assert sorted(w) == list(range(bf, bl + 1))
            slot_f = 2 * bf + (1 if sk_lo(total, G, bf) < tile * nc else 0)
            for bb, slot in w.items():
                assert slot == (slot_f if bb == bf else 2 * bb)


def _simulate(groups, runs, seed, sms=12, tokens=16):
    """Random interleavings of every CTA's roles over `runs` runs.  Per group
    (hop) h: the dequantizing warps wait for "done" (h >= 1) and, when the hop
    converts, convert (CTAs < NB) and publish; the x-tile warp waits for the
    group's "published" barrier before its x tiles when the CTA has chunks
    there; the dequantizing warps then finish the CTA's chunks of the group.
    Returns the number of scheduling steps."""
    rng = random.Random(seed)
    NB = tokens
    n_pubs = stack_plan.pubs
    hops = len(groups)
    done = pub = 0
    # per CTA, the groups in which it has chunks
    work = []
    for b in range(sms):
        w = set()
        for g in groups:
            if b < g["G"] and sk_lo(g["total"], g["G"], b + 1) > sk_lo(g["total"], g["G"], b):
                w.add(g["hidx"])
        work.append(w)
    converted = {}  # (run, hop) -> CTAs whose conversion finished
    finished = {}   # (run, hop) -> CTAs done with the hop's tasks
    steps = 0
    for run in range(runs):
        # each CTA: a generator of actions
        def cta(b):
            nonlocal done, pub
            for h in range(hops):
                if h >= 1:
                    done += 1
                    while done < (run * (hops - 1) + h) * sms:
                        yield
                    # every CTA is done with the tasks before hop h
                    assert len(finished.get((run, h - 1), ())) == sms
                head = groups[h]
                if head["conv"]:
                    if b < NB:
                        yield
                        converted.setdefault((run, head["pidx"]), set()).add(b)
                    pub += 1
                if h in work[b]:
                    while pub < (run * n_pubs + head["pidx"] + 1) * sms:
                        yield
                    # the x-tile warp copies hop h's x tiles: every conversion is published
                    assert len(converted.get((run, head["pidx"]), ())) == min(NB, sms)
                    yield
                finished.setdefault((run, h), set()).add(b)
        gens = {b: cta(b) for b in range(sms)}
        while gens:
            b = rng.choice(list(gens))
            try:
                next(gens[b])
            except StopIteration:
                del gens[b]
            steps += 1
            assert steps < 10_000_000, "deadlock"
    return steps


# small tasks leave CTAs without work in a hop: they reach the next hop's "done"
# barrier early, which a single counter for both kinds of barrier would count
# toward a "published" target (a mistake these interleavings find)
SMALL = [(2048, 1024, -1, -1), (256, 2048, 0, -1), (1024, 256, 1, -1), (2048, 1024, 2, -1), (512, 2048, 3, -1)]


@pytest.mark.parametrize("seed", range(20))
@pytest.mark.parametrize("tasks", [decode_tasks(2, h=1024, kv=256, f=2048, vocab=3072), SMALL], ids=["decode", "small"])
def test_grid_barriers_order_conversion_and_copies(seed, tasks):
    groups, _ = stack_plan(tasks, 1024, sms=12)
    _simulate(groups, runs=3, seed=seed, sms=12, tokens=8)


RING, RAW_MAX, RAW_CHUNK, A_STAGES, B_MAX = 224 * 1024, 12, 128 * 144, 3, 12


def ring_split(NB):
    """Mirror of mma_stack_create's split of the ring budget: x-tile stages
    for about 6 chunks (at least 3), the raw-chunk ring 1024-aligned after
    them with as many stages as fit."""
    b_stages = max(3, min(6, 48 * 1024 // (NB * 512)))
    raw_base = -(-b_stages * NB * 512 // 1024) * 1024
    return b_stages, raw_base, min(RAW_MAX, (RING - raw_base) // RAW_CHUNK)


@pytest.mark.parametrize("NB", [16, 32, 48, 64])
def test_ring_split(NB):
    b_stages, raw_base, raw_stages = ring_split(NB)
    assert 3 <= b_stages <= B_MAX and raw_base % 1024 == 0 and raw_base >= b_stages * NB * 512
    assert 5 <= raw_stages <= RAW_MAX and raw_base + raw_stages * RAW_CHUNK <= RING
    assert (NB * 512) % 1024 == 0  # every x stage starts on a 128-byte-swizzle atom


def test_shared_memory_budget():
    bars = 2 * RAW_MAX + 2 * A_STAGES + 2 * B_MAX + 5
    stack_smem = RING + 8 * bars + 16 + 128 + 1024
    assert stack_smem <= SMEM_OPTIN
    # the hop decision and 16 warp maxima follow the TMEM address, abort and last flags;
    # then the second accumulator's full and empty barriers (8-byte aligned)
    assert 4 * (3 + 1 + 16) == 80 and 80 + 2 * 8 <= 16 + 128


def test_two_accumulators_parities():
    """Segment k uses accumulator k % 2.  The MMA warp waits on its empty
    barrier with parity ((k >> 1) - 1) & 1 (k >= 2), the epilogue warps on its
    full barrier with parity (k >> 1) & 1; an mbarrier wait on parity p passes
    once the barrier's completion with that parity is the latest one.  Random
    interleavings: every wait passes only for the completion it means, and no
    barrier ever runs two completions ahead of a waiter (no parity aliasing)."""
    for seed in range(50):
        rng = random.Random(seed)
        n_seg = rng.randint(1, 40)
        full, empty = [0, 0], [0, 0]  # completions so far
        mma_k = epi_k = 0
        steps = 0
        while epi_k < n_seg:
            steps += 1
            assert steps < 100_000
            who = rng.choice(["mma", "epi"])
            if who == "mma" and mma_k < n_seg:
                k, a = mma_k, mma_k & 1
                if k >= 2:
                    want = (k >> 1) - 1
                    # parity wait: passes when the latest completion has parity want & 1
                    if empty[a] == 0 or (empty[a] - 1) & 1 != want & 1:
                        continue
                    assert empty[a] - 1 == want  # the completion meant, never a later one
                full[a] += 1  # MMAs of segment k, then the commit
                mma_k += 1
            elif who == "epi" and epi_k < mma_k:
                k, a = epi_k, epi_k & 1
                want = k >> 1
                if full[a] == 0 or (full[a] - 1) & 1 != want & 1:
                    continue
                assert full[a] - 1 == want
                empty[a] += 1  # read out, release
                epi_k += 1
