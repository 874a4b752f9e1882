"""The library's GGUF reader (b200q_gguf_*) and the Q4_0x8 (ggml CPU_REPACK) inverse, on the CPU.

Files are written by the installed `gguf` package (the format's own Python writer) and read back through the C ABI:
every tensor's bytes bit-identical to what was written, shapes, types and metadata as written, tensor offsets as the
package's own reader (GGUFReader) finds them; truncated and corrupt files are refused with a message. The Q4_0x8
layout is built here from its definition (ggml's block_q4_0x8 with 8-byte interleave: per 8-row group and 32-column
block the 8 fp16 scales, then chunk j of 8 quant bytes = bytes 8 (j / 8) .. of row j % 8, XOR 0x88) and read back to
the original Q4_0 rows bit for bit."""
import os

import numpy as np
import pytest

from conftest import rng

gguf = pytest.importorskip("gguf")


def to_q4_0x8(w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Q4_0 rows [rows][cols / 32 x 18] in ggml's CPU_REPACK block_q4_0x8 layout."""
    nb = cols // 32
    blk = w.reshape(rows // 8, 8, nb, 18)
    out = np.zeros((rows // 8, nb, 144), np.uint8)
    out[:, :, :16] = blk[:, :, :, :2].transpose(0, 2, 1, 3).reshape(rows // 8, nb, 16)
    qs = blk[:, :, :, 2:].transpose(0, 2, 1, 3)  # [group][block][row][16]
    for j in range(16):
        out[:, :, 16 + 8 * j:24 + 8 * j] = qs[:, :, j % 8, 8 * (j // 8):8 * (j // 8) + 8] ^ 0x88
    return out.reshape(-1)


def write_gguf(path: str, tensors: dict, meta: dict | None = None, arch: str = "b200q-test") -> None:
    """tensors: {name: (ggml type id, array)} (quantized: uint8 [rows][row bytes]; F32: float32)."""
    w = gguf.GGUFWriter(path, arch)
    for k, v in (meta or {}).items():
        if isinstance(v, str):
            w.add_string(k, v)
        elif isinstance(v, float):
            w.add_float32(k, v)
        elif isinstance(v, list):
            w.add_array(k, v)
        else:
            w.add_uint32(k, v)
    for name, (t, arr) in tensors.items():
        if t == 0:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType(t))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture
def model_file(tmp_path, synth):
    r = rng(90)
    ts = {"blk.0.ffn_gate": (2, synth.q4_0(r, 256, 512)), "blk.0.ffn_down": (8, synth.q8_0(r, 128, 1024)),
          "blk.0.ssm_out": (3, synth.q4_1(r, 96, 256)), "blk.1.ffn_up": (13, synth.q5_k(r, 64, 512)),
          "output": (14, synth.q6_k(r, 320, 768)), "output_norm": (0, r.normal(1, 0.1, 512).astype(np.float32))}
    meta = {"test.block_count": 2, "test.rope.freq_base": 1e7, "test.name": "synthetic", "test.ids": [3, 5, 8]}
    path = str(tmp_path / "m.gguf")
    write_gguf(path, ts, meta)
    return path, ts, meta


def test_tensors_read_back_bit_identical(b2, model_file):
    path, ts, meta = model_file
    ref = gguf.GGUFReader(path)
    with b2.GgufFile(path) as f:
        assert f.version == 3
        got = {t["name"]: t for t in f.tensors()}
        assert set(got) == set(ts)
        for name, (t, arr) in ts.items():
            g = got[name]
            assert g["type"] == t
            if t == 0:
                assert g["ne"] == [arr.size]
                assert np.array_equal(g["data"].view(np.float32), arr)
            else:
                rows = arr.shape[0]
                cols = arr.shape[1] // b2.gguf_row_bytes(256 if t in (13, 14) else 32, t) * (256 if t in (13, 14) else 32)
                assert g["ne"] == [cols, rows]
                assert g["bytes"] == arr.nbytes and np.array_equal(g["data"], arr.reshape(-1))
            rt = next(x for x in ref.tensors if x.name == name)
            assert g["offset"] == rt.data_offset and g["bytes"] == rt.n_bytes
        assert f.get_int("test.block_count") == 2
        assert f.get_float("test.rope.freq_base") == pytest.approx(1e7)
        assert f.get_str("test.name") == "synthetic"
        assert f.get_str("general.architecture") == "b200q-test"
        assert "test.ids" in f.keys()
        with pytest.raises(KeyError):
            f.find("missing")


def test_truncated_and_corrupt_files_are_refused(b2, model_file, tmp_path):
    path, _, _ = model_file
    blob = open(path, "rb").read()
    for cut in (3, 20, 100, len(blob) // 2, len(blob) - 7):
        p = str(tmp_path / f"cut{cut}.gguf")
        open(p, "wb").write(blob[:cut])
        with pytest.raises(b2.B200QError):
            b2.GgufFile(p)
    bad = bytearray(blob)
    bad[0:4] = b"GGUX"
    p = str(tmp_path / "magic.gguf")
    open(p, "wb").write(bytes(bad))
    with pytest.raises(b2.B200QError, match="magic"):
        b2.GgufFile(p)
    bad = bytearray(blob)
    bad[16:24] = (1 << 40).to_bytes(8, "little")  # metadata count
    p = str(tmp_path / "count.gguf")
    open(p, "wb").write(bytes(bad))
    with pytest.raises(b2.B200QError, match="count"):
        b2.GgufFile(p)
    with pytest.raises(b2.B200QError, match="cannot open"):
        b2.GgufFile(str(tmp_path / "absent.gguf"))


@pytest.mark.parametrize("rows,cols", [(8, 32), (64, 2560), (136, 4096)])
def test_q4_0x8_inverse_is_bit_exact(b2, synth, rows, cols):
    w = synth.q4_0(rng(91, rows, cols), rows, cols)
    x8 = to_q4_0x8(w, rows, cols)
    assert x8.size == w.size
    assert np.array_equal(b2.q4_0x8_to_q4_0(x8, rows, cols), w)
    with pytest.raises(b2.B200QError):
        b2.q4_0x8_to_q4_0(x8[:18 * 2], 4, 32)


def test_q4_0x8_layout_definition(synth):
    """The test's own Q4_0x8 builder against the layout's definition, spelled out for one group and block."""
    w = synth.q4_0(rng(92), 8, 32)
    x8 = to_q4_0x8(w, 8, 32)
    for r in range(8):
        assert bytes(x8[2 * r:2 * r + 2]) == bytes(w[r, :2])
        for k in range(16):
            j = 8 * (k // 8) + r
            assert x8[16 + 8 * j + k % 8] == w[r, 2 + k] ^ 0x88
