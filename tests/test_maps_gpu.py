"""Map compiler on the GPU (reference: gpu-d1/scripts/compile_corpus.py:18-95):
the device LOS table equals the native Crawl LOS table of the fixture map for all
5600 origins and the oracle's ray-fan LOS on generated maps; compiled all-pairs
distances equal the oracle BFS; a compiled map survives the corpus file round
trip unchanged."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def maps():
    from d1 import maps
    oracle.build()
    return maps


def test_los_table_equals_native_crawl_los_on_the_fixture(maps):
    z = np.load(oracle.DATA / 'fixture_1057.npz')
    m = maps.compile_map(z['floor'])
    assert np.array_equal(m.los, z['native_los'])


def test_los_table_equals_oracle_on_generated_maps(maps):
    from d1.spec_env import DEFAULT
    env = oracle.OracleSpec(3, DEFAULT, seed=21)
    floor_bits, _ = env.planes()
    for i in range(3):
        rows = floor_bits[i].reshape(70, 3)
        floor = np.array([(rows[y, x // 32] >> (x % 32)) & 1 for y in range(70) for x in range(80)], np.uint8)
        m = maps.compile_map(floor, seed=i)
        ref = np.stack([oracle.los_mask(floor, p) for p in range(5600)])
        assert np.array_equal(m.los, ref), i


def test_compiled_distances_and_file_round_trip(maps, tmp_path):
    header, kinds, floor, cells, index, distance = oracle.fixture()
    m = maps.compile_map(floor, seed=1057, hp=int(header[1]))
    # compile_corpus keeps every floor cell; the oracle BFS over the same sources
    ref = np.empty((len(m.cells), 5600), np.uint16)
    lib = oracle.library()
    assert lib.oracle_distance_table(floor.ctypes.data, m.cells.ctypes.data, len(m.cells), ref.ctypes.data) == 0
    assert np.array_equal(m.distance, ref)
    assert np.array_equal(m.index[m.cells], np.arange(len(m.cells)))
    maps.write_map(tmp_path / 'map-1057.bin', m)
    back = maps.read_corpus(tmp_path)[0]
    for k in ('floor', 'cells', 'index', 'distance', 'los'):
        assert np.array_equal(getattr(back, k), getattr(m, k)), k
    assert (back.seed, back.hp) == (1057, int(header[1]))
