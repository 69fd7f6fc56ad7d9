"""The Atlas grid and the paired batch statistics, pinned to the reference's
configs/atlas.json and bench/stats.py through tests/golden/atlas_fixture.json
(written by tests/golden/make_atlas.py)."""
import json
from pathlib import Path

import pytest

from groupconv_atlas_b200 import stats, workloads

FIXTURE = json.loads((Path(__file__).parent / 'golden' / 'atlas_fixture.json').read_text())


def test_atlas_grid_matches_reference_file():
    shapes = workloads.atlas_shapes()
    assert len(shapes) == len(FIXTURE['atlas']) == 80
    for s, ref in zip(shapes, FIXTURE['atlas']):
        assert (s.n, s.cin, s.h, s.w, s.groups) == (ref['n'], ref['cin'], ref['h'], ref['w'], ref['groups'])
        assert s.id == ref['shape_id']
        assert (s.r, s.s, s.sh, s.sw, s.ph, s.pw, s.dh, s.dw) == (3, 3, 1, 1, 1, 1, 1, 1)


@pytest.mark.parametrize('case', FIXTURE['stats'], ids=lambda c: c['compare']['classification'])
def test_compare_batches_matches_reference(case):
    got = stats.compare_batches(case['base'], case['candidate'])
    ref = case['compare']
    assert got['classification'] == ref['classification']
    assert got['paired_batches'] == ref['paired_batches']
    assert got['speedup'] == pytest.approx(ref['speedup'], rel=1e-15)
    if ref['ci95'] is None:
        assert got['ci95'] is None
    else:
        assert got['ci95'] == pytest.approx(ref['ci95'], rel=1e-15)
    d = stats.describe(case['base'])
    for key, value in case['describe_base'].items():
        assert d[key] == pytest.approx(value, rel=1e-15)


def test_classification_thresholds():
    assert stats.classify(1.06, 1.2) == 'WIN'
    assert stats.classify(0.8, 0.95) == 'LOSS'
    assert stats.classify(1 / 1.05, 1.05) == 'TIE'
    assert stats.classify(1.0, 1.1) == 'UNCERTAIN'
    assert stats.classify(0.9, 1.0) == 'UNCERTAIN'


@pytest.mark.parametrize('base,cand', [([1.0, 2.0], [1.0]), ([1.0, 0.0], [1.0, 1.0]),
                                       ([1.0, float('nan')], [1.0, 1.0]), ([], [])])
def test_compare_batches_rejects_unpaired_or_nonpositive(base, cand):
    with pytest.raises(ValueError):
        stats.compare_batches(base, cand)


def test_model_layers_match_reference_protocol():
    layers = workloads.model_layers()
    assert len(layers) == len(FIXTURE['model_layers']) == 12
    for layer, ref in zip(layers, FIXTURE['model_layers']):
        s = layer.shape
        got = dict(n=s.n, cin=s.cin, cout=s.cout, h=s.h, w=s.w, r=s.r, s=s.s, groups=s.groups, sh=s.sh, sw=s.sw,
                   ph=s.ph, pw=s.pw, dh=s.dh, dw=s.dw, bias=layer.bias, model=layer.model,
                   module_path=layer.module_path)
        assert got == {k: ref[k] for k in got}
        if not layer.bias:  # biased operations carry the reference's operation id, not a Shape id
            assert s.id == ref['shape_id']
    assert sum(layer.bias for layer in layers) == 4
