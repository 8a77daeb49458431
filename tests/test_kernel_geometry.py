"""Structural checks of the plane-pair kernel's thread geometry, on the CPU.

pla_b200/csrc/pair_kernel.cuh maps 224 threads onto a stage of two 56 x 56
planes held in shared memory as a 72 x 62 x 2 TMA box (x from -8, y from -3).
These tests restate that mapping and check, without a GPU, that every output
of the stage is owned by exactly one thread, that every shared-memory load
stays inside the box and is 8-byte aligned, that the element a tap reads is
the input the 7x7 correlation needs, and that a half-warp's 64-bit loads hit
distinct banks.  They follow the structural tests of the reference's stencil
kernels (tile coverage and alignment, data/stencil_cuda_v2/test_stencil.py:8-66).
"""
import itertools

# PairGeom<bf16> (pla_b200/csrc/pair_kernel.cuh)
S, PL, R, ELEM = 56, 2, 7, 2
RG, CG = S // R, S // 4
THREADS = PL * RG * CG
LEFT = 16 // ELEM
PITCH, ROWS = S + 2 * LEFT, S + 6


def thread_map(tid):
    pl = tid // (RG * CG)
    rem = tid - pl * RG * CG
    rg = rem // CG
    return pl, rg, rem - rg * CG


def load_offsets(tid):
    """Element offsets of the thread's three 64-bit loads for each of its 13 input rows."""
    pl, rg, cg = thread_map(tid)
    base = pl * ROWS * PITCH + (rg * R) * PITCH + 4 * cg + (LEFT - 4)
    return [[base + ir * PITCH + q for q in (0, 4, 8)] for ir in range(R + 6)]


def test_threads_and_box_shape():
    assert THREADS == 224 and THREADS % 32 == 0
    assert (PITCH * ELEM) % 16 == 0 and (LEFT * ELEM) % 16 == 0  # TMA box width and x start
    assert LEFT >= 4  # the thread's window starts 4 columns left of its first output


def test_every_output_owned_once():
    owners = {}
    for tid in range(THREADS):
        pl, rg, cg = thread_map(tid)
        for r, j in itertools.product(range(R), range(4)):
            key = (pl, rg * R + r, 4 * cg + j)
            assert key not in owners
            owners[key] = tid
    assert len(owners) == PL * S * S


def test_loads_inside_box_and_aligned():
    box = PL * ROWS * PITCH
    for tid in range(THREADS):
        for row in load_offsets(tid):
            for off in row:
                assert 0 <= off and off + 4 <= box
                assert (off * ELEM) % 8 == 0


def test_taps_read_the_correlation_inputs():
    """u[k / 2] half k & 1 is input column 4 cg - 4 + k of box row rg * 7 + ir;
    output (r, j) with tap (ky, kx) uses ir = r + ky and k = j + kx + 1."""
    for tid in range(THREADS):
        pl, rg, cg = thread_map(tid)
        base = pl * ROWS * PITCH + (rg * R) * PITCH + 4 * cg + (LEFT - 4)
        for r, j, ky, kx in itertools.product(range(R), range(4), range(7), range(7)):
            ir, k = r + ky, j + kx + 1
            assert 0 <= k < 12
            off = base + ir * PITCH + k - pl * ROWS * PITCH
            box_row, box_col = divmod(off, PITCH)
            in_row, in_col = box_row - 3, box_col - LEFT
            assert (in_row, in_col) == (rg * R + r + ky - 3, 4 * cg + j + kx - 3)


def test_half_warp_loads_hit_distinct_banks():
    for warp in range(THREADS // 32):
        for half in (0, 1):
            lanes = range(warp * 32 + 16 * half, warp * 32 + 16 * half + 16)
            for ir in range(R + 6):
                for q in range(3):
                    banks = []
                    for tid in lanes:
                        word = load_offsets(tid)[ir][q] * ELEM // 4
                        banks += [word % 32, (word + 1) % 32]
                    assert len(set(banks)) == len(banks), (warp, half, ir, q)


def test_tma_x_coordinates_stay_16_byte_aligned():
    """Every tiled TMA load of the plane kernels starts its innermost
    coordinate on a 16-byte boundary (an unaligned x is an illegal instruction
    on sm_100): plane tiles at x = tx * TW - LEFT (TileGeom, tile_kernel.cuh)
    for every element size and tile shape, and plane-pair stages at x = -LEFT."""
    for elem in (4, 2):
        left = 16 // elem
        for lx in (32, 16):            # (R, LX) = (8, 32), (7, 16), (2, 16)
            tw = 4 * lx
            pitch = tw + 2 * left
            assert (pitch * elem) % 16 == 0
            for tx in range(64):
                assert ((tx * tw - left) * elem) % 16 == 0
    assert (-LEFT * ELEM) % 16 == 0


def _stack_geom(s, mix):
    """StackGeom<S, MIX> (pla_b200/csrc/stack_kernel.cuh)."""
    r = 7 if s == 7 else 2
    rg = (s + r - 1) // r
    g = 4 if s == 7 else 1
    return r, rg, g, 32 * g


def test_stack_kernel_rows_lanes_and_stage_copies():
    """Plane-stack kernel: the (row group, row) pairs of a plane cover its S
    rows once, the lanes cover the stage's LANES planes once, every raw-stage
    read is inside the stage, 16-bit NCHW rows of even S are read as aligned
    32-bit words, and a stage is a whole number of 16-byte bulk-copy units."""
    for s in (7, 14, 28):
        for elem in (4, 2):
            mix = elem == 2
            r, rg, g, lanes = _stack_geom(s, mix)
            rows = [grp * r + i for grp in range(rg) for i in range(r) if grp * r + i < s]
            assert sorted(rows) == list(range(s))
            # The kernel's own mapping: warp = tid >> 5, lane group = warp / RG,
            # row group = warp % RG, plane lane = group * 32 + lane; every
            # (row group, plane lane) pair must belong to exactly one thread.
            warps = rg * g
            pairs = [((tid >> 5) % rg, ((tid >> 5) // rg) * 32 + (tid & 31)) for tid in range(32 * warps)]
            assert sorted(pairs) == [(a, b) for a in range(rg) for b in range(lanes)]
            plane = s * s
            stage_elems = lanes * plane
            assert (stage_elems * elem) % 16 == 0
            for ln in range(lanes):
                for iy in range(s):
                    first, last = ln * plane + iy * s, ln * plane + iy * s + s - 1   # NCHW row
                    assert 0 <= first and last < stage_elems
                    if mix and s % 2 == 0:
                        assert (first * elem) % 4 == 0
                    assert (iy * s + s - 1) * lanes + ln < stage_elems                 # NHWC row


def test_tile_kernel_covers_planes_and_reads_inside_the_box():
    """Plane-tile kernel (TileGeom, tile_kernel.cuh): for each tile shape and
    filter side, the stored outputs of all tiles cover a W x H plane once, and
    every tap of a thread reads inside the TMA box, at the input element the
    correlation needs (box x from tx * TW - LEFT, y from ty * TH - K / 2)."""
    threads = 128
    for elem in (4, 2):
        left = 16 // elem
        for r, lx in ((8, 32), (7, 16), (2, 16)):
            tw, th = 4 * lx, (threads // 32) * (32 // lx) * r
            pitch = tw + 2 * left
            for k in (3, 5, 7):
                rows = th + k - 1
                cx = 4 - k // 2
                for (h, w) in ((th, tw), (th + 5, tw + 12), (3, 8)):
                    tiles_x, tiles_y = -(-w // tw), -(-h // th)
                    seen = set()
                    for ty, tx, tid in itertools.product(range(tiles_y), range(tiles_x), range(threads)):
                        warp, lane = divmod(tid, 32)
                        rgrp, cgrp = warp * (32 // lx) + lane // lx, lane % lx
                        for rr, j in itertools.product(range(r), range(4)):
                            oy, ox = ty * th + rgrp * r + rr, tx * tw + 4 * cgrp + j
                            if oy < h and ox < w:
                                assert (oy, ox) not in seen
                                seen.add((oy, ox))
                            for ky, kx in ((0, 0), (k - 1, k - 1), (k // 2, 0), (0, k - 1)):
                                ir, col = rr + ky, j + kx + cx
                                assert 0 <= col < 12
                                box_row, box_col = rgrp * r + ir, 4 * cgrp + left - 4 + col
                                assert box_row < rows and box_col < pitch
                                assert (ty * th - k // 2 + box_row, tx * tw - left + box_col) == \
                                    (oy + ky - k // 2, ox + kx - k // 2)
                    assert len(seen) == h * w


def test_restated_constants_match_the_kernel_sources():
    """The constants and formulas restated above are read back from the
    kernel sources, so a geometry change there fails here instead of leaving
    these checks on stale numbers."""
    import os
    import re

    csrc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "pla_b200", "csrc")

    def defs(name, struct=None):
        text = open(os.path.join(csrc, name)).read()
        if struct:  # only the definitions inside `struct <name> { ... };`
            text = text[text.index(f"struct {struct} {{"):]
            text = text[:text.index("};")]
        out = {}
        for m in re.finditer(r"constexpr\s+(?:int|bool|uint32_t)\s+(\w+)\s*=\s*([^;]+);", text):
            out.setdefault(m.group(1), " ".join(m.group(2).split()))
        return out

    pair, stack, tile = defs("pair_kernel.cuh", "PairGeom"), defs("stack_kernel.cuh", "StackGeom"), \
        defs("tile_kernel.cuh", "TileGeom")
    tile["kTileThreads"] = defs("tile_kernel.cuh")["kTileThreads"]
    capi_text = open(os.path.join(csrc, "pla_capi.cu")).read()
    capi = dict(re.findall(r"\b(kWideR|kWideLX|kNarrowR|kNarrowLX|kShortR)\s*=\s*(\d+)", capi_text))
    # PairGeom
    assert (int(pair["S"]), int(pair["PL"]), int(pair["R"])) == (S, PL, R)
    assert (pair["RG"], pair["CG"], pair["THREADS"]) == ("S / R", "S / 4", "PL * RG * CG")
    assert (pair["LEFT"], pair["PITCH"], pair["ROWS"]) == ("16 / sizeof(T)", "S + 2 * LEFT", "S + 6")
    # StackGeom (_stack_geom)
    assert (stack["R"], stack["RG"], stack["G"]) == ("(S == 7) ? 7 : 2", "(S + R - 1) / R", "(S == 7) ? 4 : 1")
    assert (stack["WARPS"], stack["LANES"]) == ("RG * G", "32 * G")
    # TileGeom and the tile shapes the dispatcher instantiates
    assert int(tile["kTileThreads"]) == 128
    assert (tile["TW"], tile["TH"]) == ("4 * LX", "(kTileThreads / 32) * (32 / LX) * R")
    assert (tile["ROWS"], tile["LEFT"], tile["PITCH"]) == ("TH + K - 1", "16 / sizeof(T)", "TW + 2 * LEFT")
    shapes = {(int(capi["kWideR"]), int(capi["kWideLX"])), (int(capi["kNarrowR"]), int(capi["kNarrowLX"])),
              (int(capi["kShortR"]), int(capi["kNarrowLX"]))}
    assert shapes == {(8, 32), (7, 16), (2, 16)}

