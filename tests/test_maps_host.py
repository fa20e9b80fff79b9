"""Map file formats on the host: corpus files written here parse identically with
this package's reader and, when the reference tree is present in this container,
with the reference's own reader (gpu-d1/scripts/learn_env_v2.py:25-64); the
fixture reader agrees with the committed fixture arrays."""
import importlib.util
import pathlib
import sys

import numpy as np
import pytest

import oracle

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parents[1] / 'dcss-auto_b200'))
REF = oracle.reference_dir()


def synthetic(seed, ncells=40):
    from d1.maps import CorpusMap
    rng = np.random.default_rng(seed)
    floor = np.zeros(5600, np.uint8)
    cells = np.sort(rng.choice(5600, ncells, replace=False)).astype(np.int16)
    floor[cells] = 1
    index = np.full(5600, -1, np.int16)
    index[cells] = np.arange(ncells)
    dist = rng.integers(0, 65536, (ncells, 5600)).astype(np.uint16)
    los = rng.integers(0, 2 ** 32, (5600, 10)).astype(np.uint32)
    return CorpusMap(seed, 15, 200, 794, 906, floor, cells, index, dist, los)


def test_corpus_round_trip_and_subset_rule(tmp_path):
    from d1 import maps
    made = {s: synthetic(s) for s in (1057, 1080, 1235, 1363)}
    for s, m in made.items():
        maps.write_map(tmp_path / f'map-{s}.bin', m)
    back = maps.read_corpus(tmp_path)
    assert [m.seed for m in back] == sorted(made)
    for m in back:
        for k in ('floor', 'cells', 'index', 'distance', 'los'):
            assert np.array_equal(getattr(m, k), getattr(made[m.seed], k))
    sub = maps.read_corpus(tmp_path, map_limit=2)
    assert len(sub) == 2 and sub[0].seed == 1057
    with pytest.raises(ValueError):
        maps.read_corpus(tmp_path, map_limit=9)


@pytest.mark.skipif(not (REF / 'scripts/learn_env_v2.py').exists(), reason='reference tree not present')
def test_reference_reader_parses_files_written_here(tmp_path):
    from d1 import maps
    for s in (1057, 1589):
        maps.write_map(tmp_path / f'map-{s}.bin', synthetic(s))
    spec = importlib.util.spec_from_file_location('ref_learn_env_v2', REF / 'scripts/learn_env_v2.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    arrays, meta = mod.read_maps(tmp_path)
    ours = maps.read_corpus(tmp_path)
    for (floor, cells, index, distance, los), m, md in zip(arrays, ours, meta):
        assert md['seed'] == m.seed and md['cells'] == len(m.cells)
        assert np.array_equal(floor, m.floor) and np.array_equal(index, m.index)
        assert np.array_equal(cells[:len(m.cells)], m.cells) and (cells[len(m.cells):] == -1).all()
        assert np.array_equal(distance, m.distance.reshape(-1)) and np.array_equal(los, m.los.reshape(-1))


@pytest.mark.skipif(not (REF / 'fixtures/fixture.bin').exists(), reason='reference tree not present')
def test_fixture_reader_matches_committed_arrays():
    from d1.maps import read_fixture
    f = read_fixture(REF / 'fixtures/fixture.bin')
    z = np.load(oracle.DATA / 'fixture_1057.npz')
    for k in ('header', 'kinds', 'floor', 'native_dist', 'native_los'):
        assert np.array_equal(f[k], z[k]), k
    assert f['positions'].shape == (128,)
