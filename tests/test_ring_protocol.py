"""Host-side model of the tcgen05 kernel's K/V ring protocol (no GPU).

The kernel (csrc/moda_fwd_tc.cu) has one TMA producer and two MMA issuers (one
per query tile of a work item). This model replays the same item schedule
(causal blocks with depth blocks interleaved, fill order K_A K_B V_A V_B, a
causal block shared by both tiles filled once) and the same waits:

  producer   refills slot i only after every issuer that read the slot's
             previous fill released it;
  issuer x   per block: wait V full -> wait P -> PV (releases V) ->
             wait next K full -> S(next) (releases K).

It asserts that the protocol always drains (no circular wait) for ring depths
the kernel uses and for the shapes the tests and benchmarks run.
"""

import itertools

import pytest


def tile_info(T, L, n_tok, pair, x):
    t0 = (pair * 2 + x) * n_tok
    if t0 >= T:
        return dict(t0=t0, ndep=0, nseq=0)
    tend = min(T, t0 + n_tok)
    return dict(t0=t0, ndep=-(-(tend - t0) * L // 128), nseq=-(-tend // 128))


def item_steps(tA, tB):
    """Steps of one item, as StepWalker::next walks them."""
    S = max(tA["nseq"], tB["nseq"])
    D = max(tA["ndep"], tB["ndep"])
    j = k = 0
    out = []
    for _ in range(S + D):
        dep = k < D and (j >= S or k * S <= j * D)
        idx = k if dep else j
        if dep:
            k += 1
        else:
            j += 1
        has = [idx < (t["ndep"] if dep else t["nseq"]) for t in (tA, tB)]
        out.append((dep, idx, has))
    return out


def serpentine_items(cta, items, grid):
    """The kernel's item order for one CTA: round r covers items [r*grid, (r+1)*grid), in
    CTA order for even r and reversed for odd r; the walk stops at the first item out of
    range."""
    r = 0
    while True:
        item = r * grid + (grid - 1 - cta if r & 1 else cta)
        if item >= items:
            return
        yield item
        r += 1


def test_serpentine_order_covers_every_item_once():
    for items, grid in ((512, 148), (4096, 148), (100, 148), (1, 1), (37, 5)):
        seen = sorted(i for c in range(min(grid, items)) for i in serpentine_items(c, items, min(grid, items)))
        assert seen == list(range(items))


def build_schedule(B, Hk, T, L, G, grid):
    """Fill list (readers per fill) and per-issuer programs for CTA 0..grid-1."""
    n_tok = 128 // G
    num_pairs = -(-T // (2 * n_tok))
    items = num_pairs * B * Hk
    ctas = []
    sample = sorted({0, 1, min(grid, items) - 1})   # first, second and last CTA
    for cta in [c for c in sample if c < min(grid, items)]:
        fills = []                       # readers bitmask per fill
        progs = ([], [])                 # per tile: list of ('full', f) / ('p', blk) / ('rel', f)
        blk = [0, 0]
        for item in serpentine_items(cta, items, min(grid, items)):
            pair = num_pairs - 1 - item // (B * Hk)
            tiles = [tile_info(T, L, n_tok, pair, x) for x in (0, 1)]
            blocks = [[], []]            # per tile: (kfill, vfill)
            for dep, idx, has in item_steps(*tiles):
                shared = (not dep) and has[0] and has[1]
                kf, vf = [None, None], [None, None]
                for x in (0, 1):
                    if has[x] and not (x == 1 and shared):
                        kf[x] = len(fills)
                        fills.append(3 if shared else 1 << x)
                if shared:
                    kf[1] = kf[0]
                for x in (0, 1):
                    if has[x] and not (x == 1 and shared):
                        vf[x] = len(fills)
                        fills.append(3 if shared else 1 << x)
                if shared:
                    vf[1] = vf[0]
                for x in (0, 1):
                    if has[x]:
                        blocks[x].append((kf[x], vf[x]))
            for x in (0, 1):
                bl = blocks[x]
                if not bl:
                    continue
                prog = progs[x]
                prog += [("full", bl[0][0]), ("S", blk[x]), ("rel", bl[0][0])]
                for i, (kf, vf) in enumerate(bl):
                    prog += [("full", vf), ("p", blk[x] + i), ("rel", vf)]
                    if i + 1 < len(bl):
                        prog += [("full", bl[i + 1][0]), ("S", blk[x] + i + 1), ("rel", bl[i + 1][0])]
                blk[x] += len(bl)
        ctas.append((fills, progs))
    return ctas


def drains(fills, progs, stages):
    loaded = 0                                      # fills issued by the producer
    released = [[False, False] for _ in fills]
    pc = [0, 0]
    s_issued = [set(), set()]
    while True:
        progress = False
        # producer
        while loaded < len(fills):
            f = loaded
            if f >= stages:
                prev = f - stages
                need = fills[prev]
                if (need & 1 and not released[prev][0]) or (need & 2 and not released[prev][1]):
                    break
            loaded += 1
            progress = True
        # issuers
        for x in (0, 1):
            prog = progs[x]
            while pc[x] < len(prog):
                op, v = prog[pc[x]]
                if op == "full" and v >= loaded:
                    break
                if op == "p" and v not in s_issued[x]:   # softmax answers once S(v) exists
                    break
                if op == "S":
                    s_issued[x].add(v)
                if op == "rel":
                    released[v][x] = True
                pc[x] += 1
                progress = True
        if pc[0] == len(progs[0]) and pc[1] == len(progs[1]) and loaded == len(fills):
            return True
        if not progress:
            return False


CASES = [
    # B, Hk, T, L, G
    (4, 8, 8192, 32, 4),     # kernel-only benchmark configuration
    (2, 8, 16384, 48, 8),    # multi-GPU configuration (2 batches)
    (8, 4, 2048, 5, 2),      # module configuration
    (8, 4, 4096, 24, 4),     # model configuration
    (2, 2, 300, 32, 4),
    (1, 2, 129, 1, 2),
    (1, 2, 257, 48, 8),
    (2, 1, 1000, 5, 4),
    (1, 1, 1, 3, 1),
    (1, 1, 127, 2, 2),
    (1, 1, 256, 24, 1),
    (1, 8, 70, 48, 8),
    (1, 1, 90, 12, 1),
    (1, 1, 40, 3, 128),
    (1, 1, 200, 0, 4),
]


@pytest.mark.parametrize("stages", [4, 5, 12])
@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_ring_protocol_drains(case, stages):
    B, Hk, T, L, G = case
    for fills, progs in build_schedule(B, Hk, T, L, G, grid=148):
        assert drains(fills, progs, stages)


def test_model_catches_the_blocking_prefetch():
    """Blocking on the next K fill before the PV that frees the current V slot
    deadlocks when a tile skips steps (the last, partial tile pair)."""
    fills, progs = build_schedule(2, 2, 300, 32, 4, grid=148)[0]
    bad = []
    for prog in progs:
        out, i = [], 0
        while i < len(prog):
            op, v = prog[i]
            if op == "full" and i + 3 < len(prog) and prog[i + 1][0] == "p" and prog[i + 3][0] == "full":
                out += [prog[i], prog[i + 3], prog[i + 1], prog[i + 2]]   # prefetch next K first
                i += 4
            else:
                out.append(prog[i])
                i += 1
        bad.append(out)
    assert not drains(fills, tuple(bad), 5)
    assert drains(fills, progs, 5)
