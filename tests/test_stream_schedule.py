"""Host-side model of the attention kernel's copy stream and its cross-role
waits (dsv4_b200/csrc/sas_fwd.cu: Stream::next, the loader / MMA / softmax /
row-warp loops), run as an event simulation over random tile sequences.

The kernel's roles only ever block on the conditions modelled here, so a
sequence on which the simulation stalls is one on which the kernel would wait
until its bounded waits ran out. The test checks that no tile sequence (mixes
of 1-4 chunk tiles, segment boundaries anywhere) stalls, and that the stream
order is the same whichever role computes it.
"""

import random

import pytest

TILE_CHUNKS = 4   # TMEM score slots; chunk n uses slot n % 4
RING_SLABS = 6    # K/V slab ring
SLABS = 8         # slabs per chunk
CD = 8            # row-coordinate ring depth (chunks)
PBUF = 2          # P^T buffers


def stream_order(tile_sizes, lead=TILE_CHUNKS):
    """Stream::next: K(n) while n <= nv + 4, else V(nv) once its tile's K
    are all issued. Returns [('K'|'V', n), ...]. (`lead` other than 4 only
    for the negative control below.)"""
    last_of_tile = []
    for sz in tile_sizes:
        last_of_tile += [False] * (sz - 1) + [True]
    total = len(last_of_tile)
    nk = nv = 0
    kend = False
    out = []
    while True:
        if not kend and nk <= nv + lead:
            if nk < total:
                out.append(("K", nk))
                nk += 1
                continue
            kend = True
        if nv == nk:
            return out
        if kend or any(last_of_tile[j] for j in range(nv, nk)):
            out.append(("V", nv))
            nv += 1
            continue
        raise AssertionError("stream rule found no item")  # unreachable by construction


def simulate(tiles, seg_first_tile, lead=TILE_CHUNKS):
    """Event simulation. tiles: chunk counts; seg_first_tile[i]: tile i starts
    a segment (token). Returns True when every role finishes."""
    sizes = list(tiles)
    total = sum(sizes)
    tile_of, first_chunk = [], []
    for i, sz in enumerate(sizes):
        first_chunk.append(len(tile_of))
        tile_of += [i] * sz
    chunk_seg_first = [seg_first_tile[tile_of[n]] and n == first_chunk[tile_of[n]] for n in range(total)]
    order = stream_order(sizes, lead)
    slabs = [(kind, n, s) for kind, n in order for s in range(SLABS)]

    # state
    published = 0          # row ring: chunks published by the row warp
    loader_pos = 0         # slabs copied
    mma_pos = 0            # slabs consumed (stream position, in slabs)
    slab_freed = 0         # slabs released by the MMA
    qk_done = set()        # chunks with S^T in TMEM
    pv_done = set()        # chunks whose P.V completed
    exp_done = set()       # chunks whose exp pass wrote P
    ld_v_issued = set()    # chunks whose V copy the loaders issued
    sm_tile = 0            # softmax: next tile
    sm_chunk = 0           # softmax: next chunk within that tile
    sm_max_done = False
    epi_second_done = set()  # segments whose O^T read-out finished (O released)
    pending = []             # a read-out the softmax groups are blocked in (waiting for OFULL)
    seg_of_chunk, seg = [], -1
    for n in range(total):
        if chunk_seg_first[n]:
            seg += 1
        seg_of_chunk.append(seg)

    def cempty(n):  # coordinate slot of chunk n reusable
        return n in ld_v_issued and n in exp_done and n in pv_done

    progress = True
    while progress:
        progress = False
        # row warp: publish chunk `published` once slot (published - CD) is free
        if published < total and (published < CD or cempty(published - CD)):
            published += 1
            progress = True
        # loaders: copy slabs in stream order into the ring
        while loader_pos < len(slabs) and loader_pos - slab_freed < RING_SLABS:
            kind, n, s = slabs[loader_pos]
            if n >= published:
                break
            loader_pos += 1
            if kind == "V" and s == SLABS - 1:
                ld_v_issued.add(n)
            progress = True
        # MMA: consume in stream order, a slab at a time for K(n) (QK^T per
        # slab) and a slab pair at a time for V(n) (P.V per d-tile); an item's
        # waits are taken before its first slab
        while mma_pos < len(slabs):
            kind, n, s = slabs[mma_pos]
            if s == 0:
                if kind == "K" and n >= TILE_CHUNKS and (n - TILE_CHUNKS) not in exp_done:
                    break  # score slot n % 4: exp pass of chunk n - 4 not done
                if kind == "V":
                    if n not in exp_done:
                        break
                    if chunk_seg_first[n] and seg_of_chunk[n] > 0 and (seg_of_chunk[n] - 1) not in epi_second_done:
                        break  # O^T still being read out
            step = 2 if kind == "V" else 1
            if loader_pos < mma_pos + step:
                break
            mma_pos += step
            slab_freed += step
            if s + step == SLABS:
                (qk_done if kind == "K" else pv_done).add(n)
            progress = True
        # softmax groups
        if sm_tile < len(sizes):
            f = first_chunk[sm_tile]
            sz = sizes[sm_tile]
            if not sm_max_done:
                if all(c < published for c in range(f, f + sz)) and all(c in qk_done for c in range(f, f + sz)):
                    sm_max_done = True
                    progress = True
            if sm_max_done and sm_chunk < sz and not pending:
                n = f + sm_chunk
                ok = n < PBUF or (n - PBUF) in pv_done        # P buffer free
                ok = ok and (sm_chunk != 0 or n == 0 or (n - 1) in pv_done)  # rescale after the last P.V
                if ok:
                    exp_done.add(n)
                    sm_chunk += 1
                    progress = True
                    # the deferred O^T read-out of the previous segment runs
                    # after the first exp pass of the next segment's first tile
                    if sm_chunk == 1 and chunk_seg_first[n] and seg_of_chunk[n] > 0:
                        # blocks the softmax groups until OFULL (the
                        # previous segment's last P.V) has completed
                        pending.append(seg_of_chunk[n] - 1)
            if sm_chunk == sz and sm_max_done and not pending:
                sm_tile += 1
                sm_chunk = 0
                sm_max_done = False
                progress = True
        # pending read-outs complete once the segment's last P.V is done
        for prev in list(pending):
            last = max(c for c in range(total) if seg_of_chunk[c] == prev)
            if last in pv_done:
                epi_second_done.add(prev)
                pending.remove(prev)
                progress = True
    return published == total and mma_pos == len(slabs) and sm_tile == len(sizes) and not pending


def _random_tiles(rng, n_segs):
    tiles, firsts = [], []
    for _ in range(n_segs):
        n_win = 1
        n_cmp_tiles = rng.randint(0, 3)
        seg_tiles = [n_win] + [TILE_CHUNKS] * max(n_cmp_tiles - 1, 0) + ([rng.randint(1, 4)] if n_cmp_tiles else [])
        # a range may start inside a token: drop a prefix of its tiles
        if rng.random() < 0.2 and len(seg_tiles) > 1:
            seg_tiles = seg_tiles[rng.randint(1, len(seg_tiles) - 1):]
        for i, t in enumerate(seg_tiles):
            tiles.append(t)
            firsts.append(i == 0)
    return tiles, firsts


@pytest.mark.parametrize("seed", range(40))
def test_stream_never_stalls(seed):
    rng = random.Random(seed)
    tiles, firsts = _random_tiles(rng, rng.randint(1, 12))
    assert simulate(tiles, firsts), f"stalled on tiles={tiles} firsts={firsts}"


def test_stream_order_shape():
    # window tile then a 4-chunk tile, twice: K-first up to nv + 4
    order = stream_order([1, 4, 1, 4])
    assert order[:5] == [("K", 0), ("K", 1), ("K", 2), ("K", 3), ("K", 4)]
    # V(0) (window tile complete) comes before K(5), which needs nv >= 1
    assert order.index(("V", 0)) < order.index(("K", 5))
    # every chunk appears once as K and once as V, K first
    for n in range(10):
        assert order.index(("K", n)) < order.index(("V", n))
    assert len(order) == 20


def test_looser_rule_stalls():
    """Negative control: letting K run 6 chunks ahead (slot n % 4 still
    held by chunk n - 4, whose P.V sits behind K(n) in the ring) stalls."""
    rng = random.Random(7)
    stalled = 0
    for _ in range(40):
        tiles, firsts = _random_tiles(rng, rng.randint(2, 12))
        stalled += not simulate(tiles, firsts, lead=6)
    assert stalled > 0
