"""Quantized checkpoints (lightx2v_cuda/weights.py) in the reference's stored
layout (crates/lightx2v-core/src/export.rs:1-17, weights.rs:146-208):
written and read back bit-exactly, readable by the safetensors library and
able to read its files, and rejected with the reference's checks when
malformed."""
import json

import numpy as np
import pytest
import safetensors.numpy as stnp

from lightx2v_cuda import quant
from lightx2v_cuda.weights import SafetensorsDir, WeightsError, write_quantized


def _linears(oracle):
    return {
        "blocks.0.ffn.net.0.proj": quant.Q8.quantize(oracle.normal(81, 96 * 256, 0.02), 96, 256),
        "blocks.0.ffn.net.2": quant.Q4.quantize(oracle.normal(82, 64 * 192, 0.02), 64, 192, 64, True),
        "blocks.0.attn1.to_q": quant.Fp8E4M3.quantize(oracle.normal(83, 48 * 384, 0.02), 48, 384),
    }


def _same(a, b):
    assert type(a) is type(b)
    assert (a.rows, a.cols, a.group) == (b.rows, b.cols, b.group)
    assert np.array_equal(np.asarray(a.q).view(np.uint8), np.asarray(b.q).view(np.uint8))
    assert np.array_equal(np.asarray(a.scales, np.float32).view(np.uint32),
                          np.asarray(b.scales, np.float32).view(np.uint32))
    if isinstance(a, quant.Q4):
        assert np.array_equal(np.asarray(a.zeros, np.float32).view(np.uint32),
                              np.asarray(b.zeros, np.float32).view(np.uint32))


def test_quantized_linears_round_trip_bit_exactly(tmp_path, oracle):
    lin = _linears(oracle)
    path = str(tmp_path / "dit.safetensors")
    write_quantized(path, lin, {"lightx2v.format": "quant/1"})
    src = SafetensorsDir(path)
    for key, w in lin.items():
        assert src.has_linear(key)
        _same(src.stored(key), w)
        assert np.array_equal(src.stored(key).dequantize().view(np.uint32), w.dequantize().view(np.uint32))
    assert src.stored("blocks.0.attn1.to_k") is None
    # a directory of shards reads the same
    src_dir = SafetensorsDir(str(tmp_path))
    _same(src_dir.stored("blocks.0.ffn.net.2"), lin["blocks.0.ffn.net.2"])


def test_files_are_interchangeable_with_the_safetensors_library(tmp_path, oracle):
    lin = _linears(oracle)
    path = str(tmp_path / "ours.safetensors")
    write_quantized(path, lin)
    theirs = stnp.load_file(path)
    w8 = lin["blocks.0.ffn.net.0.proj"]
    assert np.array_equal(theirs["blocks.0.ffn.net.0.proj.weight.q8"].reshape(-1), w8.q)
    assert theirs["blocks.0.ffn.net.2.weight.q4"].shape == (64, 96)
    # and a file the library wrote reads back through ours
    other = str(tmp_path / "theirs.safetensors")
    arrs = {"k.weight.fp8": np.arange(4 * 256, dtype=np.uint8).reshape(4, 256),
            "k.weight.scale": np.linspace(0.5, 2.0, 8, dtype=np.float32).reshape(4, 2),
            "plain.weight": np.arange(6, dtype=np.float16).reshape(2, 3)}
    stnp.save_file(arrs, other)
    src = SafetensorsDir(other)
    w = src.stored("k")
    assert isinstance(w, quant.Fp8E4M3) and (w.rows, w.cols, w.group) == (4, 256, 128)
    assert np.array_equal(w.q, arrs["k.weight.fp8"].reshape(-1))
    assert np.array_equal(w.scales, arrs["k.weight.scale"].reshape(-1))
    assert np.array_equal(src.get_f32("plain.weight"), arrs["plain.weight"].astype(np.float32))


def test_bf16_tensors_read_exactly(tmp_path):
    torch = pytest.importorskip("torch")
    import safetensors.torch as stt
    t = torch.randn(5, 7).to(torch.bfloat16)
    path = str(tmp_path / "bf16.safetensors")
    stt.save_file({"x": t}, path)
    assert np.array_equal(SafetensorsDir(path).get_f32("x"), t.float().numpy())


def _write_raw(path, tensors):
    header, off, blobs = {}, 0, []
    for name, (dt, shape, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    hb = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(np.array([len(hb)], "<u8").tobytes())
        f.write(hb)
        for b in blobs:
            f.write(b)


@pytest.mark.parametrize("case", ["q8_dtype", "q8_scale_rows", "q4_zero_shape", "fp8_scale_cols", "missing_scale"])
def test_malformed_quantized_linears_are_rejected(tmp_path, case):
    path = str(tmp_path / "bad.safetensors")
    t = {}
    if case == "q8_dtype":
        t["k.weight.q8"] = ("U8", [4, 128], np.zeros((4, 128), np.uint8))
        t["k.weight.scale"] = ("F32", [4, 1], np.ones((4, 1), np.float32))
    elif case == "q8_scale_rows":
        t["k.weight.q8"] = ("I8", [4, 128], np.zeros((4, 128), np.int8))
        t["k.weight.scale"] = ("F32", [3, 1], np.ones((3, 1), np.float32))
    elif case == "q4_zero_shape":
        t["k.weight.q4"] = ("U8", [4, 64], np.zeros((4, 64), np.uint8))
        t["k.weight.scale"] = ("F16", [4, 2], np.ones((4, 2), np.float16))
        t["k.weight.zero"] = ("F16", [4, 1], np.ones((4, 1), np.float16))
    elif case == "fp8_scale_cols":
        t["k.weight.fp8"] = ("U8", [4, 128], np.zeros((4, 128), np.uint8))
        t["k.weight.scale"] = ("F32", [4, 3], np.ones((4, 3), np.float32))
    else:
        t["k.weight.fp8"] = ("U8", [4, 128], np.zeros((4, 128), np.uint8))
    _write_raw(path, t)
    with pytest.raises(WeightsError):
        SafetensorsDir(path).stored("k")
