"""Shared fixtures.  Tests marked ``gpu`` need a CUDA device (a B200) and run
the library's kernels; everything else runs on the CPU and never launches a
kernel."""
import dataclasses
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / 'tests' / 'golden'
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device and the built sm_100a library')


@pytest.fixture(scope='session')
def native():
    """The in-tree libgroupconv.so and its PyTorch front end (each rebuilt
    first when a source is newer)."""
    from groupconv_atlas_b200 import api, build
    build.build()
    build.build_torch_ext()
    return api.Native()


@pytest.fixture(scope='session')
def torch_cuda():
    torch = pytest.importorskip('torch')
    if not torch.cuda.is_available():
        pytest.skip('no CUDA device')
    return torch


@dataclasses.dataclass
class GoldenCase:
    name: str
    shape: object
    x: np.ndarray
    w: np.ndarray
    y32: np.ndarray
    y64: np.ndarray


@pytest.fixture(scope='session')
def golden_meta():
    return json.loads((GOLDEN / 'golden_meta.json').read_text())


@pytest.fixture(scope='session')
def golden_cases(golden_meta):
    from groupconv_atlas_b200.api import Shape
    data = np.load(GOLDEN / 'golden_cases.npz')
    cases = []
    for entry in golden_meta['cases']:
        name = entry['name']
        cases.append(GoldenCase(name, Shape(**entry['shape']), data[f'{name}__x'], data[f'{name}__w'],
                                data[f'{name}__y32'], data[f'{name}__y64']))
    return cases
