"""The next-token rule of the device kernels (maximum of logit / temperature, lowest index on
ties) against the reference's Sampler compiled from its sources (oracle/_ref)."""
import numpy as np
import pytest

from oracle import oracle as O


def _need_ref():
    if not O.ref_available():
        pytest.skip("reference library not built (oracle/_ref)")


@pytest.mark.parametrize("temperature", [1.0, 0.7, 1.3, 3.0, 0.05, 17.0])
@pytest.mark.parametrize("top_k", [1, 2, 4, 50, 5000])
def test_rule_matches_reference_sampler(temperature, top_k):
    _need_ref()
    rng = np.random.default_rng(int(temperature * 100) + top_k)
    for trial in range(20):
        v = int(rng.integers(2, 3000))
        row = (rng.standard_normal(v) * rng.choice([0.01, 1.0, 30.0])).astype(np.float32)
        assert O.ref_sample(row, temperature, top_k) == O.sample_rule(row, temperature)


def test_rule_on_repeated_maxima_and_infinities():
    """Exact repeats of the maximum: the reference keeps the first (its partial_sort of the
    index list puts equal scores in index order for these sizes); so does the rule."""
    _need_ref()
    row = np.zeros(64, np.float32)
    row[[5, 9, 40]] = 2.5
    for t in (1.0, 0.3):
        assert O.ref_sample(row, t, 1) == O.sample_rule(row, t) == 5
    row[[7, 11]] = np.inf
    assert O.ref_sample(row, 1.0, 1) == O.sample_rule(row, 1.0) == 7


def test_reference_sampler_config_errors():
    _need_ref()
    row = np.zeros(8, np.float32)
    with pytest.raises(ValueError, match="sampler temperature must be positive"):
        O.ref_sample(row, 0.0, 1)
    with pytest.raises(ValueError, match="sampler top_k must be positive"):
        O.ref_sample(row, 1.0, 0)
