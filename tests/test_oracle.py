"""The oracle is pinned before it is trusted: known answers from the
reference's own tests, its compiled CPU library's outputs (golden fixtures),
its Shape ids, input seeding and FP64 point selection.  CPU only."""
import json

import numpy as np
import pytest

from groupconv_atlas_b200.api import Shape, inputs
from oracle import oracle as orc


def test_pointwise_known_answer():
    # reference tests/native_cpu.cpp:38-42: 1x1 grouped conv, weights {2, 3}.
    s = Shape(n=1, cin=2, cout=2, h=2, w=3, r=1, s=1, groups=2, ph=0, pw=0)
    x = np.array([1, 2, 3, 4, 5, 6, 10, 20, 30, 40, 50, 60], np.float32).reshape(s.input)
    w = np.array([2, 3], np.float32).reshape(s.weight)
    y = orc.conv_f32_serial(s, x, w)
    assert np.array_equal(y.reshape(-1), x.reshape(-1) * np.repeat([2, 3], 6))
    # group isolation (native_cpu.cpp:43-45)
    x.reshape(-1)[6:] = 0
    assert np.all(orc.conv_f32_serial(s, x, w).reshape(-1)[6:] == 0)


def test_valid_2x2_known_answer():
    # reference tests/native_cpu.cpp:46-51: valid 2x2 cross-correlation.
    s = Shape(n=1, cin=1, cout=1, h=3, w=3, r=2, s=2, groups=1, ph=0, pw=0)
    x = np.arange(1, 10, dtype=np.float32).reshape(s.input)
    w = np.arange(1, 5, dtype=np.float32).reshape(s.weight)
    for y in (orc.conv_f32_serial(s, x, w), orc.conv_f32_blocked(s, x, w, 2), orc.conv_f64(s, x, w)):
        assert y.reshape(-1).tolist() == [37, 47, 67, 77]


def test_impulse_and_group_isolation():
    # reference tests/test_correctness.py:27-38
    s = Shape(cin=4, cout=4, groups=2, h=3, w=5)
    x = np.zeros(s.input, np.float32)
    x[0, 0, 1, 2] = 1
    w = np.ones(s.weight, np.float32)
    expected = np.zeros(s.output, np.float32)
    expected[:, :2, :, 1:4] = 1
    for y in (orc.conv_f32_serial(s, x, w), orc.conv_f32_blocked(s, x, w, 3)):
        assert np.array_equal(y, expected)


def test_hand_oracle_points():
    # reference tests/test_correctness.py:16-20
    s = Shape(cin=1, cout=1, groups=1, h=2, w=3, r=1, s=1, ph=0, pw=0)
    x = np.arange(1, 7, dtype=np.float32).reshape(s.input)
    w = np.full(s.weight, 2, np.float32)
    pos = [(0, 0, i, j) for i in range(2) for j in range(3)]
    assert np.array_equal(orc.oracle_points(s, x, w, pos), np.arange(1, 7) * 2)


def test_oracle_matches_reference_golden_bit_exact(golden_cases):
    """FP32 serial and blocked restatements reproduce the reference library's
    FP32 output bit for bit; the FP64 restatement reproduces its FP64 oracle."""
    assert len(golden_cases) >= 80
    for c in golden_cases:
        y = orc.conv_f32_serial(c.shape, c.x, c.w)
        assert np.array_equal(y.view(np.uint32), c.y32.view(np.uint32)), c.name
        yb = orc.conv_f32_blocked(c.shape, c.x, c.w, 4)
        assert np.array_equal(yb.view(np.uint32), c.y32.view(np.uint32)), c.name
        y64 = orc.conv_f64(c.shape, c.x, c.w)
        assert np.array_equal(y64, c.y64), c.name
        yv, bound = orc.conv_f64_bound(c.shape, c.x, c.w, 2)
        assert np.allclose(yv, c.y64, rtol=0, atol=1e-12), c.name
        assert np.all(bound >= np.abs(c.y64) - 1e-12), c.name


def test_golden_inputs_use_reference_seeding(golden_cases):
    """inputs() reproduces the reference's seeded generator exactly."""
    for c in golden_cases:
        if c.name.startswith('boundary'):
            x, w = inputs(c.shape, 20260908)
            assert np.array_equal(x, c.x) and np.array_equal(w, c.w), c.name


def test_shape_ids_and_point_selection(golden_meta):
    for key, sid in golden_meta['shape_ids'].items():
        s = Shape(**json.loads(key))
        assert s.id == sid
        assert [list(p) for p in orc.select_points(s, 64, 20260908)] == golden_meta['points'][sid]


def test_fp32_tolerances_against_fp64(golden_cases):
    """The reference's own FP32 output passes both acceptance checks: the
    1e-4/1e-4 gate and the sum|x*w| bound (so the bound is attainable)."""
    for c in golden_cases:
        assert orc.error_metrics(c.y32, c.y64)['passed'], c.name
        y64, bound = orc.conv_f64_bound(c.shape, c.x, c.w, 2)
        assert orc.bound_check(c.y32, y64, bound)['passed'], c.name


def test_checker_catches_planted_mistakes(golden_cases):
    """A wrong value, a NaN and a group leak planted in an oracle output are
    all rejected by the checks the GPU tests use."""
    c = next(g for g in golden_cases if g.name == 'boundary04')
    y64, bound = orc.conv_f64_bound(c.shape, c.x, c.w, 1)
    bad = c.y32.copy()
    bad.reshape(-1)[7] += 1e-3
    assert not orc.bound_check(bad, y64, bound)['passed']
    assert not orc.error_metrics(bad, c.y64)['passed']
    bad = c.y32.copy()
    bad.reshape(-1)[0] = np.nan
    assert orc.bound_check(bad, y64, bound)['failed_elements'] == 1
    assert not orc.check_points(c.shape, c.x, c.w, bad)['passed']
    for value in (np.nan, np.inf, -np.inf):
        assert not orc.error_metrics(np.array([value]), np.array([0.0]))['passed']


@pytest.mark.skipif(not orc.reference_available(), reason='reference library not built here')
def test_oracle_matches_reference_library_random():
    """Cross-check on fresh random shapes against the compiled reference."""
    rng = np.random.default_rng(5)
    for _ in range(12):
        cpg = int(rng.choice([1, 2, 3, 4, 8]))
        g = int(rng.integers(1, 4))
        s = Shape(n=int(rng.integers(1, 3)), cin=cpg * g, cout=cpg * g * int(rng.integers(1, 3)),
                  h=int(rng.integers(1, 20)), w=int(rng.integers(1, 24)), groups=g,
                  r=int(rng.choice([1, 3, 5])), s=int(rng.choice([1, 3])), ph=1, pw=1)
        if min(s.output) <= 0:
            continue
        x, w = inputs(s, int(rng.integers(1 << 30)))
        for impl in (0, 1, 2):
            ref = orc.reference_conv(s, x, w, impl=impl, threads=2)
            assert np.array_equal(orc.conv_f32_blocked(s, x, w, 2).view(np.uint32), ref.view(np.uint32))
