"""The reference's Sampler::sample (compiled from its sources into oracle/_ref) against the numpy restatement with
the seed's uniform draw as input: pins that the draw is u x (the kept candidates' sum), which the device sampler
takes as its input."""
import numpy as np
import pytest

from tests.sampler_restatement import sample

PARAMS = [(0.8, 40, 0.95, 1.1, 64), (1.0, 1, 1.0, 1.0, 0), (0.7, 1024, 0.9, 1.3, 32), (1.5, 0, 0.5, 1.0, 64),
          (0.0, 40, 0.95, 1.1, 64)]


@pytest.mark.parametrize("params", PARAMS)
def test_reference_sampler_is_the_restatement_with_its_draw(params):
    from oracle.oracle import Reference
    R = Reference()
    rng = np.random.default_rng(3)
    for case in range(12):
        V = 1000 if case % 2 else 5000
        x = (rng.standard_normal(V) * 3).astype(np.float32)
        hist = rng.integers(0, V, 40).tolist() + [int(np.argmax(x))] * 3
        seed = 1000 + case
        want, _ = R.sample(x, hist, *params, seed)
        got = sample(x, hist, *params, R.sampler_draw(seed))
        assert got == want, (params, case)
