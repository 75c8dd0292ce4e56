"""The sampling step without a GPU: the generator (XoshiroRandom), the oracle's
restatement of the reference samplers against the cases of the reference's own
tests (tests/DotNetFoundryLLM.Sampling.Tests), and fl_sample's argument checks.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from dotnetfoundryllm_b200 import _native as N
from dotnetfoundryllm_b200.runtime import XoshiroRandom
from oracle import oracle as O


def test_splitmix64_known_answer():
    # the first SplitMix64 output of seed 0 (the algorithm's published value)
    assert XoshiroRandom(0).s[0] == 0xE220A8397B1DCDAF
    assert int(O.Xoshiro(0).state[0]) == 0xE220A8397B1DCDAF


@pytest.mark.parametrize("seed", [0, 1, 7, 42, 123, 999, (1 << 63) + 5])
def test_python_generator_equals_the_restatement(seed):
    py, c = XoshiroRandom(seed), O.Xoshiro(seed)
    for _ in range(500):
        assert py.next_uint64() == c.next_uint64()
    for _ in range(2000):
        u = py.next_float()
        assert u == c.next_float()
        assert 0.0 <= u <= 1.0


def test_top_p_keeps_the_nucleus():
    # TopPSamplerTests.ApplyTopP_SmallP_ZeroesOutLowProbTokens
    p = O.apply_topp(np.array([0.02, 0.90, 0.05, 0.03], np.float32), 0.91)
    assert p[0] == 0.0 and p[1] > 0.0 and p[2] > 0.0 and p[3] == 0.0
    # ApplyTopP_RenormalizesRemainingProbabilities
    q = O.apply_topp(np.array([0.1, 0.6, 0.2, 0.1], np.float32), 0.8)
    assert abs(float(q.sum()) - 1.0) < 1e-5
    # ApplyTopP_P1_LeavesDistributionUnchanged
    r = O.apply_topp(np.array([0.1, 0.6, 0.2, 0.1], np.float32), 1.0)
    np.testing.assert_allclose(r, [0.1, 0.6, 0.2, 0.1], atol=1e-5)


def test_pipeline_cases_of_the_reference_tests():
    # SamplerPipelineTests.Sample_ZeroTemperature_Greedy
    assert O.sampler_pipeline(np.array([0.1, 5.0, 3.0], np.float32), 0.0, 0, 1.0, 0.5)[0] == 1
    # Sample_TopK1_AlwaysReturnsArgmax
    rng = O.Xoshiro(42)
    for _ in range(20):
        assert O.sampler_pipeline(np.array([1, 10, 0.5, 3], np.float32), 1.0, 1, 1.0, rng.next_float())[0] == 1
    # Sample_IsDeterministicWithSameSeed
    a, b = O.Xoshiro(123), O.Xoshiro(123)
    lg = np.array([0.5, 0.3, 0.9, 0.1], np.float32)
    for _ in range(50):
        assert O.sampler_pipeline(lg, 1.0, 0, 1.0, a.next_float())[0] == O.sampler_pipeline(lg, 1.0, 0, 1.0,
                                                                                            b.next_float())[0]
    # Sample_AlwaysReturnsValidIndex
    rng = O.Xoshiro(7)
    for _ in range(100):
        t = O.sampler_pipeline(np.array([0.1, 0.5, 0.3, 0.1], np.float32), 1.0, 2, 0.9, rng.next_float())[0]
        assert 0 <= t < 4


def test_temperature_one_samples_uniform_logits_evenly():
    # TemperatureSamplerTests: four equal logits, each token ~1/4 of 2000 draws
    rng = O.Xoshiro(5)
    counts = np.zeros(4, int)
    for _ in range(2000):
        counts[O.sampler_pipeline(np.ones(4, np.float32), 1.0, 0, 1.0, rng.next_float())[0]] += 1
    assert np.all((counts / 2000 > 0.17) & (counts / 2000 < 0.33))


def test_repetition_penalty():
    # RepetitionPenaltySamplerTests: 5.0 / 1.5 < 4.0, so greedy moves to token 2
    lg = O.apply_repetition_penalty(np.array([0.1, 5.0, 4.0], np.float32), [1], 1.5)
    assert O.sampler_pipeline(lg, 0.0, 0, 1.0, 0.0)[0] == 2
    # negative logits are multiplied; each occurrence applies again
    lg = O.apply_repetition_penalty(np.array([-2.0, 3.0, 1.0], np.float32), [0, 1, 1, 7], 2.0)
    np.testing.assert_array_equal(lg, np.array([-4.0, 3.0 / 2.0 / 2.0, 1.0], np.float32))


def test_fl_sample_rejects_bad_arguments_before_device_work():
    lib = N.cuda()
    d = N.FlSamplerDesc(C.sizeof(N.FlSamplerDesc), 1.0, 0, 1.0, 1.0)
    tok = C.c_int32()
    assert lib.fl_sample(None, C.byref(d), None, 0, 0.5, C.byref(tok)) == N.FL_ERR_ARG
    assert lib.fl_sample(C.c_void_p(256), None, None, 0, 0.5, C.byref(tok)) == N.FL_ERR_ARG
