"""Pin the optimizer side of the oracle against the reference's own compiled code.

The golden trajectory in tests/golden/optimizer.npz was produced by the reference's
src/train_optimizer.h (oracle/_ref/libsa3ref.so); the inverse_lr constants are the ones the
reference's tests/train_optimizer_test.cpp:35-47 quotes from the Python trainer.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_adamw_restatement_matches_reference_trajectory():
    g = np.load(os.path.join(GOLD, "optimizer.npz"))
    lr, b1, b2, eps, wd = (float(v) for v in g["hp"])
    p = g["p0"].copy()
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    for step in range(1, 7):
        oracle.adamw_f32(p, g["grads"][step - 1], m, v, lr, b1, b2, eps, wd, step)
        ref_p, ref_m, ref_v = g["traj"][step - 1]
        np.testing.assert_array_max_ulp(p, ref_p, maxulp=2)
        np.testing.assert_array_max_ulp(m, ref_m, maxulp=2)
        np.testing.assert_array_max_ulp(v, ref_v, maxulp=2)


def test_inverse_lr_reference_quotes():
    g = np.load(os.path.join(GOLD, "optimizer.npz"))
    quoted = g["quoted_inverse_lr"]
    assert len(quoted) == 7
    # the compiled reference reproduces its own test's quoted values (rel < 1e-5)
    for (step, lr), got in zip(quoted, g["inv_lr"][: len(quoted)]):
        assert abs(got - lr) / lr < 1e-5


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
def test_reference_adamw_sign_and_errors():
    # tests/train_optimizer_test.cpp:18-31
    ref = oracle.ref()
    p = np.array([1.0, -1.0], np.float32)
    gr = np.array([0.5, -0.25], np.float32)
    m = np.zeros(2, np.float32)
    v = np.zeros(2, np.float32)
    err = ctypes.create_string_buffer(128)
    assert ref.sa3ref_adamw_update(oracle._ptr(p), oracle._ptr(gr), oracle._ptr(m), oracle._ptr(v),
                                   2, 0.1, 0.9, 0.999, 1e-8, 0.01, 1, err, 128) == 0
    assert p[0] < 1.0 and p[1] > -1.0
    assert ref.sa3ref_adamw_update(oracle._ptr(p), oracle._ptr(gr), oracle._ptr(m), oracle._ptr(v),
                                   2, 0.1, 0.9, 0.999, 1e-8, 0.01, 0, err, 128) == 1
    assert b"step must be positive" in err.value


def test_average_and_clip_semantics():
    # src/train_loop.h:147-171: mean over count, f64 global norm, scale when norm > clip
    a = np.full(4, 3.0, np.float32)
    b = np.full(4, 4.0, np.float32)
    norm = oracle.average_and_clip([a, b], 2, 1.0)
    assert np.isclose(norm, np.sqrt(4 * 1.5 ** 2 + 4 * 2.0 ** 2))
    assert np.isclose(np.sqrt((a ** 2).sum() + (b ** 2).sum()), 1.0, rtol=1e-5)
    c = np.full(4, 0.1, np.float32)
    norm = oracle.average_and_clip([c], 1, 1.0)
    assert np.allclose(c, 0.1)                     # below the clip: untouched


def test_diffusion_sample_matches_reference():
    g = np.load(os.path.join(GOLD, "diffusion.npz"))
    t = np.float32(g["t"])
    z, n = g["z"], g["noise"]
    xt = (np.float32(1) - t) * z + t * n
    assert np.array_equal(xt, g["x_t"])
    assert np.array_equal(n - z, g["v"])


def test_package_sample_at_matches_reference_diffusion():
    import train_inputs
    g = np.load(os.path.join(GOLD, "diffusion.npz"))
    xt, v = train_inputs.sample_at(g["z"], g["t"], g["noise"])
    assert np.array_equal(xt, g["x_t"]) and np.array_equal(v, g["v"])


def test_package_expo_features_matches_restatement():
    import train_inputs
    for t in (0.0, 0.3, 0.999):
        a = train_inputs.expo_features(t, 256, 0.5, 10000.0)
        b = oracle.expo_features(t, 256, 0.5, 10000.0)
        np.testing.assert_allclose(a, b, rtol=0, atol=2e-6)
