"""Map files of the reference and their compiler on the GPU.

* fixture.bin -- the single-map fixture (writer gpu-d1/scripts/compile_fixture.py:
  75-80, reader learn_env.py:15-40): magic 0x44314750, 8-int header (player, hp,
  ac100, ev100, sh100, shield_limit, regen, 0), 6 monster kinds x 4 ints, floor
  u8[5600], distance from the player u16[5600], native LOS masks u32[5600, 10],
  64 contact + 64 approach cells i16.
* map-SEED.bin -- one map of a corpus (writer compile_corpus.py:88-95, reader
  learn_env_v2.py:25-64): magic 0x44325650, seed, ncells (u32), hp, ac100,
  ev100, sh100 (i32), floor u8[5600], cells i16[5600] (-1 padded), index
  i16[5600], all-pairs distance u16[ncells, 5600], LOS masks u32[5600, 10].

compile_map() builds a map's tables on the device: cells/index on the host
(a prefix over 5600 bytes), the all-pairs BFS with learn_distance_table (one warp
per source) and the LOS masks with d1_los_table (one warp per origin, the env
step's ray evaluation) -- replacing the reference's Python BFS and per-origin ray
loop. The file layout is kept byte-for-byte so the reference's readers load it.
"""
import hashlib
import pathlib
import struct
from dataclasses import dataclass

import numpy as np

N, W, H = 5600, 80, 70
FIXTURE_MAGIC, CORPUS_MAGIC = 0x44314750, 0x44325650


def read_fixture(path):
    raw = pathlib.Path(path).read_bytes()
    if struct.unpack_from('<I', raw)[0] != FIXTURE_MAGIC:
        raise ValueError(f'{path}: not a fixture map')
    header = np.array(struct.unpack_from('<8i', raw, 4), np.int32)
    kinds = np.array(struct.unpack_from('<24i', raw, 36), np.int32).reshape(6, 4)
    off = 132
    floor = np.frombuffer(raw, np.uint8, N, off).copy(); off += N
    dist = np.frombuffer(raw, '<u2', N, off).copy(); off += 2 * N
    los = np.frombuffer(raw, '<u4', N * 10, off).copy().reshape(N, 10); off += 40 * N
    positions = np.frombuffer(raw, '<i2', 128, off).copy() if len(raw) >= off + 256 else None
    return dict(header=header, kinds=kinds, floor=floor, native_dist=dist, native_los=los, positions=positions)


@dataclass
class CorpusMap:
    seed: int
    hp: int
    ac100: int
    ev100: int
    sh100: int
    floor: np.ndarray      # u8 [5600]
    cells: np.ndarray      # i16 [ncells]
    index: np.ndarray      # i16 [5600]
    distance: np.ndarray   # u16 [ncells, 5600]
    los: np.ndarray        # u32 [5600, 10]
    name: str = ''

    def to_bytes(self):
        n = len(self.cells)
        cells = np.full(N, -1, '<i2')
        cells[:n] = self.cells
        return b''.join([struct.pack('<3I', CORPUS_MAGIC, self.seed, n),
                         struct.pack('<4i', self.hp, self.ac100, self.ev100, self.sh100),
                         np.ascontiguousarray(self.floor, np.uint8).tobytes(), cells.tobytes(),
                         np.ascontiguousarray(self.index, '<i2').tobytes(),
                         np.ascontiguousarray(self.distance, '<u2').tobytes(),
                         np.ascontiguousarray(self.los, '<u4').tobytes()])


def parse_map(raw, name=''):
    magic, seed, ncells = struct.unpack_from('<3I', raw)
    if magic != CORPUS_MAGIC or ncells > N:
        raise ValueError(f'bad corpus map: {name}')
    hp, ac, ev, sh = struct.unpack_from('<4i', raw, 12)
    off = 28
    floor = np.frombuffer(raw, np.uint8, N, off).copy(); off += N
    cells = np.frombuffer(raw, '<i2', N, off).copy()[:ncells]; off += 2 * N
    index = np.frombuffer(raw, '<i2', N, off).copy(); off += 2 * N
    distance = np.frombuffer(raw, '<u2', ncells * N, off).copy().reshape(ncells, N); off += 2 * ncells * N
    los = np.frombuffer(raw, '<u4', N * 10, off).copy().reshape(N, 10)
    return CorpusMap(seed, hp, ac, ev, sh, floor, cells, index, distance, los, name)


def write_map(path, m):
    path = pathlib.Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_bytes(m.to_bytes())
    return hashlib.sha256(path.read_bytes()).hexdigest()


def read_corpus(root, map_limit=None):
    """All map-*.bin of a corpus directory (or its `all/` subdirectory), in seed
    order. With map_limit, a nested subset that does not depend on the run seed:
    the first map, then the others ordered by the SHA-256 of their file names
    (the selection rule of learn_env_v2.py:36-45)."""
    def key(p):
        try:
            return (0, int(p.stem.split('-', 1)[1]))
        except (IndexError, ValueError):
            return (1, p.name)

    root = pathlib.Path(root)
    paths = sorted(root.glob('map-*.bin'), key=key)
    if not paths and (root / 'all').is_dir():
        paths = sorted((root / 'all').glob('map-*.bin'), key=key)
    if map_limit is not None:
        if not 1 <= map_limit <= len(paths):
            raise ValueError(f'map_limit must be 1..{len(paths)}')
        rest = sorted(paths[1:], key=lambda p: hashlib.sha256(p.name.encode()).digest())
        paths = sorted((paths[:1] + rest)[:map_limit], key=key)
    if not paths:
        raise ValueError('corpus must contain at least one map')
    return [parse_map(p.read_bytes(), p.name) for p in paths]


def compile_map(floor, seed=0, hp=15, ac100=200, ev100=794, sh100=906, device='cuda'):
    """Build a corpus map's tables for a u8[5600] floor on the GPU."""
    import torch
    from ._lib import check, library, launch_stream
    from .spec_env import device_rays
    lib = library()
    dev = torch.device(device)
    floor = np.ascontiguousarray(floor, np.uint8).reshape(N)
    cells = np.flatnonzero(floor).astype(np.int16)
    index = np.full(N, -1, np.int16)
    index[cells] = np.arange(len(cells), dtype=np.int16)
    f = torch.from_numpy(floor).to(dev)
    c = torch.from_numpy(cells).to(dev)
    dist = torch.empty((len(cells), N), dtype=torch.int16, device=dev)
    los = torch.empty((N, 10), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        device_rays(dev)
        s = launch_stream(dev)
        if len(cells):
            check(lib.learn_distance_table(f.data_ptr(), c.data_ptr(), len(cells), dist.data_ptr(), s),
                  'learn_distance_table')
        check(lib.d1_los_table(f.data_ptr(), los.data_ptr(), s), 'd1_los_table')
    return CorpusMap(seed, hp, ac100, ev100, sh100, floor, cells, index,
                     dist.cpu().numpy().view(np.uint16), los.cpu().numpy().view(np.uint32))
