"""The adapter / trainer-state GGUF files (src/train_checkpoint.h:42-173, src/train_resume.h) on
the host: our writer read back by the independent `gguf` package (the ggml project's Python GGUF
reader), and files written by that package's writer read by ours.  No GPU needed: the library
loads without one and these entry points are host code."""
import os

import numpy as np
import pytest

import sa3k

gguf = pytest.importorskip("gguf")


def test_adapter_file_matches_reference_layout(tmp_path):
    """The reference test's fixture (tests/train_checkpoint_test.cpp:20-46): rank 2, alpha 4, one
    3 -> 5 target; A and B hold 0, 1, 2, ... row-major."""
    path = str(tmp_path / "adapter.gguf")
    A = np.arange(6, dtype=np.float32).reshape(2, 3)      # [rank][in]
    B = np.arange(10, dtype=np.float32).reshape(5, 2)     # [out][rank]
    sa3k.adapter_gguf_write(path, "lora", 2, 4.0, [("dit.0.self.qkv", A, B, None)])
    r = gguf.GGUFReader(path)
    kv = {f.name: f for f in r.fields.values()}
    assert kv["general.architecture"].contents() == "sa3-lora"
    assert kv["general.name"].contents() == "sa3 native trained adapter"
    assert kv["lora.adapter_type"].contents() == "lora"
    assert kv["lora.rank"].contents() == 2 and kv["lora.rank"].types == [gguf.GGUFValueType.UINT32]
    assert kv["lora.alpha"].contents() == 4.0 and kv["lora.alpha"].types == [gguf.GGUFValueType.FLOAT32]
    assert kv["lora.n_targets"].contents() == 1
    t = {x.name: x for x in r.tensors}
    assert sorted(t) == ["dit.0.self.qkv.lora_A", "dit.0.self.qkv.lora_B"]
    # ggml dims ne[0] innermost: A ne {in, rank} = {3, 2}, B ne {rank, out} = {2, 5}
    assert list(t["dit.0.self.qkv.lora_A"].shape) == [3, 2]
    assert list(t["dit.0.self.qkv.lora_B"].shape) == [2, 5]
    assert t["dit.0.self.qkv.lora_A"].tensor_type == gguf.GGMLQuantizationType.F32
    np.testing.assert_array_equal(np.asarray(t["dit.0.self.qkv.lora_A"].data).ravel(), A.ravel())
    np.testing.assert_array_equal(np.asarray(t["dit.0.self.qkv.lora_B"].data).ravel(), B.ravel())
    # and our own reader
    a, ne = sa3k.gguf_get_f32(path, "dit.0.self.qkv.lora_A")
    assert ne == (3, 2)
    np.testing.assert_array_equal(a, A.ravel())
    assert sa3k.gguf_get_string(path, "lora.adapter_type") == "lora"
    assert sa3k.gguf_get_u64(path, "lora.rank") == 2
    assert not os.path.exists(path + ".tmp")


def test_dora_adapter_file_has_magnitudes(tmp_path):
    path = str(tmp_path / "dora.gguf")
    rng = np.random.default_rng(0)
    targets = []
    for stem, i, o in (("dit.0.ff.out", 64, 32), ("dit.0.self.out", 32, 32)):
        targets.append((stem, rng.standard_normal((4, i)).astype(np.float32),
                        rng.standard_normal((o, 4)).astype(np.float32), rng.random(o).astype(np.float32)))
    sa3k.adapter_gguf_write(path, "dora-rows", 4, 4.0, targets)
    r = gguf.GGUFReader(path)
    t = {x.name: x for x in r.tensors}
    assert len(t) == 6
    for stem, A, B, m in targets:
        np.testing.assert_array_equal(np.asarray(t[stem + ".magnitude"].data).ravel(), m)
        assert list(t[stem + ".magnitude"].shape) == [m.size]
        np.testing.assert_array_equal(np.asarray(t[stem + ".lora_A"].data).ravel(), A.ravel())
        np.testing.assert_array_equal(np.asarray(t[stem + ".lora_B"].data).ravel(), B.ravel())
    # every tensor starts on the 32-byte alignment of the format
    for x in r.tensors:
        assert x.data_offset % 32 == 0


def test_reader_reads_independent_writer(tmp_path):
    """A trainer-state style file written by the gguf package is read by our metadata / tensor
    readers (string, u32, u64, u64 array, string array skipped, f32 tensors)."""
    path = str(tmp_path / "state.gguf")
    w = gguf.GGUFWriter(path, "sa3-trainer-state")
    w.add_string("trainer.compatibility", "test-compatibility")
    w.add_uint32("trainer.state_version", 1)
    w.add_uint64("trainer.step", 3)
    w.add_key_value("trainer.order", [1, 0, 7], gguf.GGUFValueType.ARRAY, sub_type=gguf.GGUFValueType.UINT64)
    w.add_array("trainer.targets", ["dit.0.self.qkv"])
    m = np.linspace(-1, 1, 12, dtype=np.float32)
    w.add_tensor("optimizer.dit.0.self.qkv.lora_A.m", m)
    w.add_tensor("two_d", np.arange(6, dtype=np.float32).reshape(2, 3))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    assert sa3k.gguf_get_string(path, "general.architecture") == "sa3-trainer-state"
    assert sa3k.gguf_get_string(path, "trainer.compatibility") == "test-compatibility"
    assert sa3k.gguf_get_u64(path, "trainer.state_version") == 1
    assert sa3k.gguf_get_u64(path, "trainer.step") == 3
    assert sa3k.gguf_get_u64_array(path, "trainer.order") == [1, 0, 7]
    v, ne = sa3k.gguf_get_f32(path, "optimizer.dit.0.self.qkv.lora_A.m")
    np.testing.assert_array_equal(v, m)
    v2, ne2 = sa3k.gguf_get_f32(path, "two_d")
    assert ne2 == (3, 2)
    np.testing.assert_array_equal(v2, np.arange(6, dtype=np.float32))
    with pytest.raises(sa3k.Sa3kError):
        sa3k.gguf_get_u64(path, "trainer.compatibility")     # a string, not an integer
    with pytest.raises(sa3k.Sa3kError):
        sa3k.gguf_get_f32(path, "missing")


def test_reader_rejects_truncated_and_foreign_files(tmp_path):
    path = str(tmp_path / "a.gguf")
    sa3k.adapter_gguf_write(path, "lora", 2, 4.0, [("x", np.ones((2, 3), np.float32), np.ones((5, 2), np.float32),
                                                   None)])
    data = open(path, "rb").read()
    cut = str(tmp_path / "cut.gguf")
    open(cut, "wb").write(data[: len(data) - 40])
    with pytest.raises(sa3k.Sa3kError):
        sa3k.gguf_get_f32(cut, "x.lora_B")           # tensor data runs past the end
    foreign = str(tmp_path / "foreign.bin")
    open(foreign, "wb").write(b"NOTGGUF" + bytes(64))
    with pytest.raises(sa3k.Sa3kError):
        sa3k.gguf_get_string(foreign, "general.architecture")
