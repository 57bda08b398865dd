"""The INT4 checkpoint tool's file handling (clove_compute_b200/quantize.py), on the
CPU: its safetensors reader and writer agree with the reference implementation of
the format (the `safetensors` package) in both directions, reject malformed files,
and select the weights the tool packs."""
import os
import struct

import numpy as np
import pytest

from clove_compute_b200 import quantize as q

safetensors_np = pytest.importorskip("safetensors.numpy")


def _sample():
    rng = np.random.default_rng(0)
    return {
        "layers.0.mlp.up.weight": rng.standard_normal((256, 512)).astype(np.float16),
        "layers.0.mlp.up.bias": rng.standard_normal(256).astype(np.float32),
        "embed.weight": rng.standard_normal((10, 128)).astype(np.float32),
        "step": np.array(7, dtype=np.int64),
        "mask": np.array([True, False, True]),
        "empty": np.zeros((0, 128), dtype=np.float16),
        "codes": rng.integers(0, 256, (3, 5), dtype=np.uint8),
    }


def test_written_files_read_by_the_reference_package(tmp_path):
    arrs = _sample()
    p = str(tmp_path / "a.safetensors")
    q.write_safetensors(p, {k: q.Tensor.from_numpy(v) for k, v in arrs.items()}, {"k": "v"})
    back = safetensors_np.load_file(p)
    assert set(back) == set(arrs)
    for k, v in arrs.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        np.testing.assert_array_equal(back[k], v)
    (n,) = struct.unpack("<Q", open(p, "rb").read(8))
    assert n % 8 == 0  # tensor data starts 8-byte aligned


def test_reads_files_of_the_reference_package(tmp_path):
    arrs = _sample()
    p = str(tmp_path / "b.safetensors")
    safetensors_np.save_file(arrs, p, metadata={"format": "np"})
    tensors, meta = q.read_safetensors(p)
    assert meta == {"format": "np"}
    assert set(tensors) == set(arrs)
    for k, v in arrs.items():
        np.testing.assert_array_equal(tensors[k].numpy(), v)


def test_bf16_weights_are_widened_exactly(tmp_path):
    vals = np.array([[1.0, -2.5, 0.15625, 65280.0]], dtype=np.float32)
    bits = (vals.view(np.uint32) >> 16).astype(np.uint16)  # exact bf16 values
    t = q.Tensor("BF16", (1, 4), bits.tobytes())
    np.testing.assert_array_equal(q._to_fp16(t), vals.astype(np.float16))


@pytest.mark.parametrize("corrupt", ["short", "header_len", "offsets"])
def test_malformed_files_rejected(tmp_path, corrupt):
    p = str(tmp_path / "c.safetensors")
    q.write_safetensors(p, {"w": q.Tensor.from_numpy(np.ones((4, 4), np.float32))})
    raw = bytearray(open(p, "rb").read())
    if corrupt == "short":
        raw = raw[:5]
    elif corrupt == "header_len":
        raw[:8] = struct.pack("<Q", len(raw) * 2)
    else:
        raw = raw[:-4]  # the tensor's bytes end early
    open(p, "wb").write(bytes(raw))
    with pytest.raises(ValueError):
        q.read_safetensors(p)


def test_selection():
    f16 = lambda shape: q.Tensor.from_numpy(np.zeros(shape, np.float16))
    assert q.selects("mlp.up.weight", f16((256, 512)), r".")
    assert not q.selects("mlp.up.bias", f16((256,)), r".")            # 1-D
    assert not q.selects("odd.weight", f16((256, 200)), r".")          # K % 128
    assert not q.selects("mlp.up.weight", f16((256, 512)), r"attn")    # filtered out
    assert not q.selects("ids", q.Tensor.from_numpy(np.zeros((4, 128), np.int32)), r".")
    assert q.selects("w", q.Tensor("BF16", (2, 128), bytes(512)), r".")
