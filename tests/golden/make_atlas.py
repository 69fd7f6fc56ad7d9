"""Generate the fixture that pins the Atlas grid and the batch statistics.

Run in a checkout where the reference tree is available (it is read, never
copied):

    python tests/golden/make_atlas.py --reference <reference checkout>

It writes ``atlas_fixture.json`` next to this script:

  atlas   per shape of the reference's configs/atlas.json: n, cin, h, w,
          groups and the reference's shape id, in the file's order.
  stats   paired batch-median inputs and the reference's own
          bench/stats.py compare_batches / describe results for them.
  model_layers  the reference's 12 frozen model-layer operations
          (configs/model-shapes-protocol.json): geometry, bias flag, model,
          module path and shape id.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_stats(reference):
    spec = importlib.util.spec_from_file_location('ref_stats', Path(reference) / 'bench' / 'stats.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--reference', required=True)
    args = parser.parse_args()
    atlas = json.loads((Path(args.reference) / 'configs' / 'atlas.json').read_text())
    shapes = [{k: s[k] for k in ('n', 'cin', 'h', 'w', 'groups', 'shape_id')} for s in atlas['shapes']]
    ref = load_stats(args.reference)
    rng = np.random.default_rng(7)
    cases = []
    # (batches, base centre, candidate centre, relative spread)
    for batches, base, cand, spread in [(5, 100.0, 80.0, 0.02), (10, 100.0, 80.0, 0.02), (10, 100.0, 99.0, 0.01),
                                        (10, 100.0, 120.0, 0.02), (12, 50.0, 48.5, 0.05), (10, 10.0, 10.2, 0.2),
                                        (15, 7.0, 3.0, 0.1)]:
        b = (base * (1 + spread * rng.standard_normal(batches))).round(4).tolist()
        c = (cand * (1 + spread * rng.standard_normal(batches))).round(4).tolist()
        cases.append({'base': b, 'candidate': c, 'compare': ref.compare_batches(b, c),
                      'describe_base': ref.describe(b)})
    proto = json.loads((Path(args.reference) / 'configs' / 'model-shapes-protocol.json').read_text())
    keys = ('n', 'cin', 'cout', 'h', 'w', 'r', 's', 'groups', 'sh', 'sw', 'ph', 'pw', 'dh', 'dw', 'bias', 'model',
            'module_path', 'shape_id')
    layers = [{k: s[k] for k in keys} for s in proto['frozen_shapes']]
    out = {'source': 'configs/atlas.json, configs/model-shapes-protocol.json and bench/stats.py of the reference',
           'atlas': shapes, 'stats': cases, 'model_layers': layers}
    (HERE / 'atlas_fixture.json').write_text(json.dumps(out, indent=1) + '\n')
    print(f'{len(shapes)} shapes, {len(cases)} statistics cases, {len(layers)} model layers')


if __name__ == '__main__':
    main()
