"""The boundary from compiled code, without a GPU: include/sa3k.h compiles as C and
include/sa3_train.h as C++ against the built library (prototypes checked by the compilers, not
by name), and the host side of the training API reproduces the reference's seeded draws:
  - TrainDiffusionSampler (src/train_diffusion.h:50-125): t and noise streams of both timestep
    modes bit-identical to the reference's own sampler compiled from its header (oracle/_ref),
    and x_t / v = (1 - t) z + t n, n - z;
  - init_train_lora_state (src/train_lora.h:205-273): A of every target bit-identical to the
    restated std::mt19937_64 + uniform_real_distribution<float> draw (oracle/stdrng.py, itself
    pinned by the C++ standard's mt19937_64 known answer), B = 0, targets in name order."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

import host_programs
import stdrng


@pytest.fixture(scope="module")
def cpu_run(tmp_path_factory):
    d = tmp_path_factory.mktemp("train_api_cpu")
    exe = host_programs.build("train_api.cpp", str(d))
    r = subprocess.run([exe, "cpu", str(d)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    return d


def test_c_abi_compiles_as_c(tmp_path):
    host_programs.build("abi_linear.c", str(tmp_path))


def test_mt19937_64_known_answer():
    e = stdrng.MT19937_64()
    for _ in range(9999):
        e()
    assert e() == 9981545732273789042


def test_lora_init_matches_seeded_draw(cpu_run):
    order = (cpu_run / "init_order.txt").read_text().split()
    assert order == sorted(order)
    shapes = {"dit.0.self.qkv.weight": (96, 64), "dit.0.ff.proj.weight": (64, 160), "dit.1.self.out.weight": (128, 64),
              "dit.proj_in.weight": (64, 64)}
    ref = np.concatenate(stdrng.lora_init_A(987654321, [shapes[n] for n in order], 4))
    got = np.fromfile(cpu_run / "init_lora_A.f32", np.float32)
    assert np.array_equal(got, ref)
    assert not np.any(np.fromfile(cpu_run / "init_lora_B.f32", np.float32))


@pytest.mark.parametrize("mode", ["uniform", "trunc_logit_normal"])
def test_sampler_matches_reference(cpu_run, mode):
    import oracle
    if not oracle.ref_available():
        pytest.skip("the reference's compiled sampler (oracle/_ref) is not built")
    z = np.array([0.5, -1.0, 2.0, 0.25, -0.75, 1.5, 0.0], np.float32)
    n_steps = 5
    t_ref = np.zeros(n_steps, np.float32)
    noise_ref = np.zeros(n_steps * z.size, np.float32)
    fn = oracle.ref().sa3ref_diffusion_stream
    fn.argtypes = [ctypes.c_ulonglong, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_long, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p]
    assert fn(20240611, mode.encode(), z.ctypes.data, z.size, n_steps, t_ref.ctypes.data, noise_ref.ctypes.data) == 0
    t = np.fromfile(cpu_run / f"sampler_{mode}_t.f32", np.float32)
    noise = np.fromfile(cpu_run / f"sampler_{mode}_noise.f32", np.float32)
    assert np.array_equal(t, t_ref) and np.array_equal(noise, noise_ref)
    xt = np.fromfile(cpu_run / f"sampler_{mode}_xt.f32", np.float32).reshape(n_steps, -1)
    v = np.fromfile(cpu_run / f"sampler_{mode}_v.f32", np.float32).reshape(n_steps, -1)
    nz = noise.reshape(n_steps, -1)
    one = np.float32(1.0)
    assert np.array_equal(xt, (one - t[:, None]) * z[None] + t[:, None] * nz)
    assert np.array_equal(v, nz - z[None])
