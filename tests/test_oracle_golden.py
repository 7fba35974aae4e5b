"""The oracle reproduces every known answer of the reference's own tests
(pins the CPU restatement before it is trusted as the checker)."""
import numpy as np
import pytest

from _golden import check, run_oracle
from conftest import golden_cases


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_kat(orc, case):
    check(case, run_oracle(case))


def test_relu_negative_gives_negative_zero(orc):
    # ReLU is x & map(x > 0 ? 1 : 0) (activation/relu.rs:36-41): -2 * 0 = -0.0
    x = orc.contiguous(np.array([-2.0, 0.0, 3.0], dtype=np.float32))
    y = orc.unary("relu", x)
    assert np.signbit(y[0]) and y[0] == 0.0
    assert y[2] == 3.0


def test_max_axis_nan_rules(orc):
    # strict `>` from the first element (base.rs:1404-1411): NaN sticks only at index 0
    x = orc.contiguous(np.array([[np.nan, 1.0, 2.0], [1.0, np.nan, 2.0], [2.0, 2.0, 1.0]], dtype=np.float32))
    v, i = orc.max_argmax_axis(x, 1)
    assert np.isnan(v[0]) and i[0] == 0
    assert v[1] == 2.0 and i[1] == 2
    assert v[2] == 2.0 and i[2] == 0


def test_sum_is_a_sequential_f32_fold(orc):
    # sum (base.rs:1024-1030) folds left to right in f32: 1e8 + 1 + ... stays 1e8
    x = orc.contiguous(np.array([1e8] + [1.0] * 16, dtype=np.float32))
    assert orc.sum_all(x) == np.float32(1e8)


def test_elu_large_positive_is_nan(orc):
    # ELU::forward computes (e^x - 1) * alpha * 0 for x > 0, which is inf * 0 = NaN past x ~ 88.7
    x = orc.contiguous(np.array([100.0, 1.0, -1.0], dtype=np.float32))
    y = orc.unary("elu", x, 1.0)
    assert np.isnan(y[0]) and y[1] == 1.0 and y[2] < 0


def test_storage_indices_negative_stride(orc):
    st = np.arange(6, dtype=np.int32)
    v = orc.HostView(st, [6], [-1], 5)
    assert orc.unary("none", v).tolist() == [5, 4, 3, 2, 1, 0]


def test_integer_division_by_zero_panics(orc):
    a = orc.contiguous(np.array([1, 2], dtype=np.int32))
    b = orc.contiguous(np.array([1, 0], dtype=np.int32))
    with pytest.raises(orc.OracleError):
        orc.binary("div", a, b)


def test_seeded_uniform_is_exact_in_f32(orc):
    u = orc.fill_uniform(np.float32, 1 << 16, seed=0)
    d = orc.fill_uniform(np.float64, 1 << 16, seed=0)
    assert np.array_equal(u.astype(np.float64), d)
    assert u.min() >= -1.0 and u.max() < 1.0
