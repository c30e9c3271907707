"""Adapter and trainer-state files of the DiT training state on the GPU: the reference's exact
continuation contract (tests/train_checkpoint_test.cpp:48-124: uninterrupted AdamW equals
checkpoint + reload + continue), immutable checkpoint pairs, the adapter fingerprint binding and
the adapter round trip."""
import os

import numpy as np
import pytest

import test_gpu_dit as T

pytestmark = pytest.mark.gpu


def _steps(dit, inputs, first, n):
    import sa3k
    hp = sa3k.AdamWParams(1e-3, 0.9, 0.95, 1e-8, 0.01, 1.0)
    for s in range(first, first + n):
        dit.zero_grads()
        dit.forward_backward(T.B, T.T, T.CTX, *inputs)
        dit.apply_adamw(T.B, hp, s)


def _params(dit, which=0):
    out = np.zeros(dit.size(), np.float32)
    dit.copy(which, out, to_model=False)
    return out


def test_checkpoint_continuation_matches_uninterrupted(ctx, tmp_path):
    import sa3k
    cfg = dict(T.CFG)
    dit, deq, ad, targets, rng = T._build(ctx, cfg, seed=3)
    inputs = T._inputs(rng)
    _steps(dit, inputs, 1, 3)
    a, s = str(tmp_path / "adapter-step-3.gguf"), str(tmp_path / "trainer-state-step-3.gguf")
    dit.save_checkpoint(a, s, 3, epoch=2, next_sample=1, order=(1, 0), compatibility="test-compatibility",
                        rng={"shuffle": "123 456", "diffusion": "789"})
    with pytest.raises(sa3k.Sa3kError, match="overwrite"):
        dit.save_checkpoint(a, s, 3, order=(1, 0))
    _steps(dit, inputs, 4, 3)
    uninterrupted = _params(dit)
    dit.close()

    fresh, _, _, _, rng2 = T._build(ctx, cfg, seed=3)
    assert fresh.load_checkpoint(a, s) == 3
    assert sa3k.gguf_get_u64(s, "trainer.epoch") == 2 and sa3k.gguf_get_u64(s, "trainer.next_sample") == 1
    assert sa3k.gguf_get_u64_array(s, "trainer.order") == [1, 0]
    assert sa3k.gguf_get_string(s, "trainer.compatibility") == "test-compatibility"
    assert sa3k.gguf_get_string(s, "trainer.rng.shuffle") == "123 456"
    assert sa3k.gguf_get_string(s, "trainer.adapter_file") == "adapter-step-3.gguf"
    _steps(fresh, inputs, 4, 3)
    continued = _params(fresh)
    # the same gradients up to the order of f32 atomic additions, through bit-exact AdamW
    assert T.rel_l2(continued, uninterrupted) < 1e-5

    # a changed adapter file no longer matches its trainer state
    bad = str(tmp_path / "tampered.gguf")
    data = bytearray(open(a, "rb").read())
    data[-1] ^= 1
    open(bad, "wb").write(bytes(data))
    with pytest.raises(sa3k.Sa3kError, match="does not match its trainer-state"):
        fresh.load_checkpoint(bad, s)
    fresh.close()


def test_adapter_file_round_trip_and_checks(ctx, tmp_path):
    import sa3k
    cfg = dict(T.CFG)
    dit, deq, ad, targets, rng = T._build(ctx, cfg, seed=4)
    path = str(tmp_path / "adapter.gguf")
    dit.save_adapter(path)
    saved = _params(dit)
    # layout: <stem>.lora_A ne {in, rank}, <stem>.lora_B ne {rank, out}, <stem>.magnitude ne {out}
    for i, name in enumerate(targets):
        oa, ob, om = dit.offsets(i)
        stem = name[:-len(".weight")]
        A, neA = sa3k.gguf_get_f32(path, stem + ".lora_A")
        Bm, neB = sa3k.gguf_get_f32(path, stem + ".lora_B")
        mag, neM = sa3k.gguf_get_f32(path, stem + ".magnitude")
        out, inn = ad[name]["B"].shape[0], ad[name]["A"].shape[1]
        assert neA == (inn, T.RANK) and neB == (T.RANK, out) and neM == (out,)
        np.testing.assert_array_equal(A, saved[oa:oa + A.size])
        np.testing.assert_array_equal(Bm, saved[ob:ob + Bm.size])
        np.testing.assert_array_equal(mag, saved[om:om + out])
    assert sa3k.gguf_get_string(path, "lora.adapter_type") == "dora-rows"
    other, *_ = T._build(ctx, cfg, seed=5)
    assert T.rel_l2(_params(other), saved) > 1e-2
    other.load_adapter(path)
    np.testing.assert_array_equal(_params(other), saved)
    other.close()
    # a plain-LoRA model refuses a DoRA adapter file, a model with other targets refuses it too
    lora, *_ = T._build(ctx, cfg, seed=5, adapter="lora")
    with pytest.raises(sa3k.Sa3kError, match="type/rank/alpha"):
        lora.load_adapter(path)
    lora.close()
    core, *_ = T._build(ctx, cfg, seed=5, scope="core")
    with pytest.raises(sa3k.Sa3kError, match="target count"):
        core.load_adapter(path)
    core.close()
    dit.close()
