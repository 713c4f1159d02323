"""CPU checks of the tensor-core GEMV stack (gemm_q4_0_mma_stack_kernel,
nexusllm_b200/csrc/mma_stack_kernels.cuh; mma_stack_create in nexus_gpu.cu),
restated in Python before any GPU run:

* the host plan: which tasks are hops (a new input, or an `after` task not yet
  behind a barrier), each task's hop index and stream-K CTA count;
* every task's chunks are covered once by its CTAs' ranges, and the CTAs the
  fix-up counts for a shared tile (sk_owner of its first and last chunk) are
  exactly the CTAs that work on it, so a grow-only arrival counter marks
  exactly one last arrival per tile in every run;
* the two grid barrier counters, simulated with many random interleavings of
  the CTAs' roles over several runs: no conversion starts before every CTA is
  done with the tasks before its hop, no x tile is copied before every CTA
  published its conversion, and nothing deadlocks;
* the shared-memory budget of the kernel.
"""
import random

import pytest

from tests.test_mma_plan import SMEM_BYTES, sk_lo, sk_owner, tc_ctas

ROWS, RAW_K = 128, 256
SMS = 148
SMEM_OPTIN = 232448


def stack_plan(tasks, input_cols, sms=SMS):
    """tasks: (rows, cols, x_source, after).  Mirror of mma_stack_create:
    hops, hop index, stream-K CTAs, group position, and the x slot (0: the
    stack input, converted at its first hop of a run; 1: an earlier task's y,
    converted at every hop) with the "published" barrier that covers it."""
    plan, hops, last_hop, gpos = [], 0, 0, 0
    pubs, in_pub, cur_pub = 0, -1, -1
    for i, (rows, cols, src, after) in enumerate(tasks):
        assert cols % RAW_K == 0
        assert (input_cols if src < 0 else tasks[src][0]) == cols
        hop = i == 0 or src != tasks[i - 1][2] or (after >= 0 and after >= last_hop)
        if hop:
            hops += 1
            last_hop = i
            gpos = 0
        tiles = -(-rows // ROWS)
        nc = cols // RAW_K
        total = tiles * nc
        conv = hop and (src >= 0 or in_pub < 0)
        if conv:
            cur_pub = pubs
            pubs += 1
            if src < 0:
                in_pub = cur_pub
        plan.append(dict(rows=rows, cols=cols, tiles=tiles, nc=nc, total=total,
                         G=tc_ctas(sms, tiles, nc), hop=hop, hidx=hops - 1, gpos=gpos,
                         conv=conv, pidx=in_pub if src < 0 else cur_pub, xslot=0 if src < 0 else 1))
        gpos += 1
    stack_plan.pubs = pubs
    return plan, hops


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
    plan, hops = stack_plan(decode_tasks(3), 4096)
    assert [p["hop"] for p in plan[:7]] == [True, False, False, True, True, False, True]
    assert hops == 4 * 3 + 1  # q, o, gate, down per layer; the head reads the stack input again
    for i, p in enumerate(plan):
        assert p["hidx"] == sum(q["hop"] for q in plan[:i + 1]) - 1
    # the stack input is converted once (q of layer 0); o, gate and down convert every layer
    assert [p["conv"] for p in plan[:14]] == [True, False, False, True, True, False, True,
                                             False, False, False, True, True, False, True]
    assert stack_plan.pubs == 1 + 3 * 3 and not plan[-1]["conv"]
    assert all(plan[i]["pidx"] == 0 and plan[i]["xslot"] == 0 for i in (0, 7, len(plan) - 1))
    # a task's "published" barrier is its own group's conversion, or the stack input's
    for i, p in enumerate(plan):
        last_conv = max(j for j in range(i + 1) if plan[j]["conv"] and plan[j]["xslot"] == p["xslot"])
        assert p["pidx"] == plan[last_conv]["pidx"]
    # an `after` on the previous task with the same input forces a hop
    plan, hops = stack_plan([(256, 256, -1, -1), (256, 256, -1, 0)], 256)
    assert plan[1]["hop"] and hops == 2


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336), (128256, 4096),
                                       (300, 256), (128, 256), (1, 512), (8192, 28672)])
def test_stream_k_cover_and_fixup_arrivals(rows, cols):
    plan, _ = stack_plan([(rows, cols, -1, -1)], cols)
    p = plan[0]
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


def test_partial_slots_are_never_shared_within_a_hop_group():
    """Tasks of one hop group run with no barrier between them: a CTA's
    partial-sum slots for its shared tiles (2 per task: its range's first and
    last tile) must differ across the group's tasks, and the slots the fix-up
    reads for a tile are the ones its CTAs wrote."""
    plan, _ = stack_plan(decode_tasks(2), 4096)
    n_slots = 2 * (max(p["gpos"] for p in plan) + 1)
    assert n_slots == 6  # q, k, v
    for b in range(SMS):
        used = {}
        for t, p in enumerate(plan):
            G, nc, total = p["G"], p["nc"], p["total"]
            if b >= G:
                continue
            lo, hi = sk_lo(total, G, b), sk_lo(total, G, b + 1)
            t0, t1 = lo // nc, (hi - 1) // nc
            for tile in range(t0, t1 + 1):
                c0 = lo - tile * nc if tile == t0 else 0
                c1 = hi - tile * nc if tile == t1 else nc
                if c0 == 0 and c1 == nc:
                    continue
                slot = 2 * p["gpos"] + (0 if tile == t0 else 1)
                assert slot < n_slots
                key = (p["hidx"], slot)
                assert key not in used, (b, t, tile, used.get(key))
                used[key] = (t, tile)
                # the fix-up's slot for CTA b of this tile
                assert 2 * p["gpos"] + (0 if tile == sk_lo(total, G, b) // nc else 1) == slot


def _simulate(plan, hops, runs, seed, sms=12, tokens=16):
    """Random interleavings of every CTA's roles over `runs` runs.  Per hop h:
    the dequantizing warps wait for "done" (h >= 1) and, when the hop converts,
    convert (CTAs < NB) and publish; the x-tile warp waits for the hop's
    "published" barrier before the x tiles of a task in hop h when the CTA has
    chunks there; the dequantizing warps then finish the CTA's tasks of hop h.
    Returns the number of scheduling steps."""
    rng = random.Random(seed)
    NB = tokens
    n_pubs = stack_plan.pubs
    hop_task = [next(p for p in plan if p["hidx"] == h) for h in range(hops)]
    done = pub = 0
    # per CTA, the hops in which it has chunks
    work = []
    for b in range(sms):
        w = set()
        for p in plan:
            if b < min(p["G"], sms) and sk_lo(p["total"], min(p["G"], sms), b + 1) > sk_lo(p["total"], min(p["G"], sms), b):
                w.add(p["hidx"])
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
                head = hop_task[h]
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
    plan, hops = stack_plan(tasks, 1024, sms=12)
    _simulate(plan, hops, runs=3, seed=seed, sms=12, tokens=8)


def test_shared_memory_budget():
    stack_smem = SMEM_BYTES + 128
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
