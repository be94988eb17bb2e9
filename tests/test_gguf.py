"""GGUF ingestion (include/mlq.h mlq_gguf_*) against the reference's own
GGUF reader (src/gguf.cc compiled into oracle/_ref/libref_gguf.so): the same
files accepted and rejected, the same tensor table and data offset, the
same tensor bytes.  Files come from tests/gguf_writer.py.  The device upload
is tested in tests/test_gguf_gpu.py; here only its argument checks."""
from __future__ import annotations

import struct

import numpy as np
import pytest

import gguf_writer as gw

Q80, Q40, Q41, F32, F16 = 8, 2, 3, 0, 1


@pytest.fixture(scope="module")
def ref_gguf():
    from oracle.oracle import ReferenceGguf
    if not ReferenceGguf.available():
        pytest.skip("reference GGUF reader oracle/_ref/libref_gguf.so not built here")
    return ReferenceGguf()


def _model_file(oracle, pkg, alignment=None):
    meta = [("general.architecture", gw.STRING, "llama"), ("llama.block_count", gw.U32, 2),
            ("llama.context_length", gw.U64, 4096), ("llama.rope.freq_base", gw.F32, 500000.0),
            ("llama.attention.layer_norm_rms_epsilon", gw.F64, 1e-5), ("flag", gw.BOOL, 1),
            ("small", gw.I8, -3), ("u16", gw.U16, 65535), ("i16", gw.I16, -2), ("i64", gw.I64, -(1 << 40)),
            ("tokenizer.ggml.tokens", gw.ARRAY, (gw.STRING, ["a", "bc", ""])),
            ("tokenizer.ggml.scores", gw.ARRAY, (gw.F32, [0.5, -1.0])),
            ("nested", gw.ARRAY, (gw.ARRAY, [(gw.U8, [1, 2]), (gw.STRING, ["x"])]))]
    tensors = [("blk.0.ffn_up.weight", [256, 96], Q80, gw.quantized(oracle, "q8_0", 96, 256, 1, pkg.synth)),
               ("blk.0.ffn_down.weight", [96, 256], Q40, gw.quantized(oracle, "q4_0", 256, 96, 2, pkg.synth)),
               ("blk.0.attn_q.weight", [128, 40], Q41, gw.quantized(oracle, "q4_1", 40, 128, 3, pkg.synth)),
               ("blk.0.attn_norm.weight", [256], F32, np.arange(256, dtype=np.float32).tobytes()),
               ("token_embd.weight", [64, 3], F16, np.ones(192, np.float16).tobytes()),
               ("odd.type", [32], 7, b"")]
    return gw.build(meta, tensors, alignment=alignment), tensors


@pytest.mark.parametrize("alignment", [None, 64, 4096])
def test_table_and_bytes_match_reference(tmp_path, oracle, pkg, ref_gguf, alignment):
    raw, tensors = _model_file(oracle, pkg, alignment)
    path = tmp_path / "m.gguf"
    path.write_bytes(raw)
    ok, err, doff, rtab, rdata = ref_gguf.load(path)
    assert ok, err
    with pkg.mlq.GgufFile(path) as g:
        assert g.data_offset == doff
        tab = g.tensors()
        assert [{k: t[k] for k in ("name", "dims", "type", "offset")} for t in tab] == rtab
        for i, t in enumerate(tab):
            if t["nbytes"]:
                start = doff + t["offset"]
                assert raw[start:start + t["nbytes"]] == rdata[i]  # the bytes the upload copies
            else:
                assert rdata[i] == b""  # a type neither reader sizes
        assert g.find("blk.0.ffn_down.weight") == 1 and g.find("missing") == -1
        up = tab[0]
        assert (up["rows"], up["row_bytes"]) == (96, 8 * 34)
        assert g.metadata_int("llama.block_count") == 2
        assert g.metadata_int("llama.context_length") == 4096
        assert g.metadata_int("i64") == -(1 << 40) and g.metadata_int("small") == -3
        assert g.metadata_int("flag") == 1 and g.metadata_int("u16") == 65535
        assert g.metadata_float("llama.rope.freq_base") == 500000.0
        assert g.metadata_float("llama.attention.layer_norm_rms_epsilon") == 1e-5
        with pytest.raises(pkg.mlq.MLQError):
            g.metadata_int("general.architecture")  # a string
        with pytest.raises(pkg.mlq.MLQError):
            g.metadata_int("absent")


def _bad_files(oracle, pkg):
    q = gw.quantized(oracle, "q4_0", 4, 64, 5, pkg.synth)
    good_t = [("w", [64, 4], Q40, q)]
    yield "magic", gw.build([], good_t, magic=b"GGUG")
    yield "version 2", gw.build([], good_t, version=2)
    yield "repeated key", gw.build([("k", gw.U32, 1), ("k", gw.U32, 2)], good_t)
    yield "repeated tensor", gw.build([], good_t + [("w", [64, 4], Q40, q)])
    yield "zero dim", gw.build([], [("w", [64, 0], Q40, b"")])
    yield "nine dims", gw.build([], [("w", [1] * 9, F32, b"\0" * 4)])
    yield "alignment 48", gw.build([], good_t, alignment=48)
    yield "alignment 0", gw.build([], good_t, alignment=0)
    yield "data past end", gw.build([], good_t, pad_data=False, truncate=1)
    yield "partial block", gw.build([], [("w", [48], Q80, b"\0" * 51)])
    yield "bad value type", (b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 1) + b"k" +
                             struct.pack("<I", 13) + b"\0" * 64)
    # header only: a truncated string length
    yield "truncated", b"GGUF" + struct.pack("<IQQ", 3, 1, 1) + struct.pack("<Q", 100) + b"ab"


def test_rejects_what_the_reference_rejects(tmp_path, oracle, pkg, ref_gguf):
    for name, raw in _bad_files(oracle, pkg):
        path = tmp_path / (name.replace(" ", "_") + ".gguf")
        path.write_bytes(raw)
        ok, err, *_ = ref_gguf.load(path)
        with pytest.raises(pkg.mlq.MLQError) as e:
            pkg.mlq.GgufFile(path)
        assert not ok, (name, "the reference accepted it")
        assert e.value.status in (1, 9), (name, e.value.status)


def test_upload_argument_checks(tmp_path, oracle, pkg):
    """Row range, destination size and tensor type are checked before any
    CUDA call (no GPU needed)."""
    raw, _ = _model_file(oracle, pkg)
    path = tmp_path / "m.gguf"
    path.write_bytes(raw)
    mlq = pkg.mlq
    with mlq.GgufFile(path) as g:
        with pytest.raises(mlq.MLQError) as e:
            g.upload_rows(0, 0, 97, 0x1000, 1 << 20)  # past the 96 rows
        assert e.value.status == 9
        with pytest.raises(mlq.MLQError) as e:
            g.upload_rows(0, 0, 96, 0x1000, 96 * 272 - 1)  # destination one byte short
        assert e.value.status == 9 and b"need" in mlq.lib().mlq_last_error()
        with pytest.raises(mlq.MLQError) as e:
            g.upload_rows(5, 0, 1, 0x1000, 64)  # a type without a size
        assert e.value.status == 1
        with pytest.raises(mlq.MLQError) as e:
            g.upload_rows(0, 0, 96, None, 1 << 20)
        assert e.value.status == 2
