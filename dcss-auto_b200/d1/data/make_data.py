#!/usr/bin/env python3
"""Convert the reference's map fixture and native LOS ray fan into compact arrays.

Run once in a container that has the reference tree; the outputs are committed so
that nothing at run time needs the reference checkout:

  python dcss-auto_b200/d1/data/make_data.py /path/to/reference/gpu-d1

fixture_1057.npz
    The only real D:1 map the reference ships (gpu-d1/fixtures/fixture.bin, written
    by gpu-d1/scripts/compile_fixture.py:75-80): header (player, hp, ac100, ev100,
    sh100, shield_limit, regen, 0), six monster kinds (speed, damage, to-hit,
    bypass), the 80x70 floor bytes, the native distance field from the fixture's
    player cell (used to pick reachable cells exactly as
    gpu-d1/scripts/learn_env.py:22 does) and the native 17x17 LOS masks
    (10 x u32 per origin), kept only as a golden vector for the LOS kernel.

los_rays.npz
    Crawl's LOS ray fan for one quadrant as exported natively
    (gpu-d1/fixtures/native-1057.rays, parsed the same way as
    gpu-d1/scripts/compile_corpus.py:56-63). Only cellrays that end inside the
    8x8 quadrant survive: the native export marks the radius-8 row and column as
    outside, so the view is the 15x15 square. Each ray becomes (end_x, end_y,
    blockers) where blockers is a 64-bit mask over the quadrant cells (bit y*8+x)
    whose opacity kills the ray.
"""
import os
import pathlib
import struct
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def convert_fixture(ref: pathlib.Path):
    raw = (ref / 'fixtures/fixture.bin').read_bytes()
    assert struct.unpack_from('<I', raw)[0] == 0x44314750, 'not a D:1 fixture'
    header = np.array(struct.unpack_from('<8i', raw, 4), np.int32)
    kinds = np.array(struct.unpack_from('<24i', raw, 36), np.int32).reshape(6, 4)
    floor = np.frombuffer(raw, np.uint8, 5600, 132).copy()
    native_dist = np.frombuffer(raw, '<u2', 5600, 5732).copy()
    los = np.frombuffer(raw, '<u4', 56000, 5732 + 11200).reshape(5600, 10).copy()
    np.savez_compressed(HERE / 'fixture_1057.npz', header=header, kinds=kinds, floor=floor,
                        native_dist=native_dist, native_los=los)


def convert_rays(ref: pathlib.Path):
    lines = (ref / 'fixtures/native-1057.rays').read_text().splitlines()
    count = int(lines[0])
    ends = [tuple(map(int, lines[1 + i].split())) for i in range(count)]
    through = {}
    for line in lines[1 + count:]:
        x, y, inside, bits = line.split()
        if int(inside):
            through[(int(x), int(y))] = int(bits[::-1], 2)
    inside_cells = set(through)
    assert inside_cells == {(x, y) for x in range(8) for y in range(8)}, 'view is not 15x15'
    rows = []
    for i, (ex, ey) in enumerate(ends):
        if (ex, ey) not in inside_cells:
            continue
        mask = 0
        for (x, y), bits in through.items():
            if (bits >> i) & 1:
                assert (x, y) != (ex, ey), 'a ray must not be blocked by its own end cell'
                mask |= 1 << (y * 8 + x)
        rows.append((ex, ey, mask))
    ex = np.array([r[0] for r in rows], np.int32)
    ey = np.array([r[1] for r in rows], np.int32)
    blockers = np.array([r[2] for r in rows], np.uint64)
    np.savez_compressed(HERE / 'los_rays.npz', end_x=ex, end_y=ey, blockers=blockers)
    return len(rows)


if __name__ == '__main__':
    # The reference's gpu-d1 folder: the argument, else $DCSS_REFERENCE/gpu-d1.
    if len(sys.argv) > 1:
        ref = pathlib.Path(sys.argv[1])
    elif os.environ.get('DCSS_REFERENCE'):
        ref = pathlib.Path(os.environ['DCSS_REFERENCE']) / 'gpu-d1'
    else:
        sys.exit('usage: make_data.py <reference gpu-d1 folder> (or set DCSS_REFERENCE)')
    convert_fixture(ref)
    print('rays kept:', convert_rays(ref))
