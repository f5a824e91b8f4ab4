"""GGUF ingest on the host (no GPU): the C++ reader (host/gguf.cpp) against
the reference's own parser test (src/gguf/reader.zig "parseBytes: synthetic
GGUF v3"), files written by llmtoy-zig_b200/gguf.py, the info report
(src/main.zig:520-618) and malformed inputs."""
from __future__ import annotations

import importlib
import struct

import numpy as np
import pytest

from conftest import REPO


def _mods():
    return (importlib.import_module("llmtoy-zig_b200.decoder"), importlib.import_module("llmtoy-zig_b200.gguf"),
            importlib.import_module("llmtoy-zig_b200.synth"))


def _reference_test_bytes() -> bytes:
    """The byte image built by reader.zig's parse test: GGUF v3, one f32 4x4
    tensor "weight", general.architecture = "test_arch",
    test.context_length = 256 (u32), data at the 32-byte boundary."""
    s = lambda x: struct.pack("<Q", len(x)) + x.encode()  # noqa: E731
    b = struct.pack("<IIQQ", 0x46554747, 3, 1, 2)
    b += s("general.architecture") + struct.pack("<I", 8) + s("test_arch")
    b += s("test.context_length") + struct.pack("<II", 4, 256)
    b += s("weight") + struct.pack("<IQQIQ", 2, 4, 4, 0, 0)
    b += b"\0" * ((-len(b)) % 32)
    return b + b"\0" * 64


def test_reference_parse_test(tmp_path):
    decoder, _, _ = _mods()
    p = tmp_path / "ref.gguf"
    p.write_bytes(_reference_test_bytes())
    with decoder.GgufFile(p) as g:
        info = g.info()
        assert "version:   GGUF v3" in info
        assert "metadata:  2 entries" in info
        assert "tensors:   1" in info
        assert "arch:      test_arch" in info
        assert g.tensors() == [("weight", 0, 64)]  # 16 f32 elements


def test_model_file_round_trip(tmp_path):
    decoder, gguf, synth = _mods()
    m = synth.DecoderModel(np.random.default_rng(3), 2, 256, 4, 2, 64, 500, n_experts=8, k=2, d_expert=256,
                           lm_type=14, qk_norm=True, rope_neox=True, norm_topk=True)
    p = gguf.write_model(tmp_path / "m.gguf", m)
    meta, ts = gguf.model_tensors(m, "qwen3moe")
    with decoder.GgufFile(p) as g:
        got = g.tensors()
        assert [n for n, _, _ in got] == [t[0] for t in ts]
        for (n, t, nb), (_, t2, _, data) in zip(got, ts):
            assert t == t2 and nb == np.asarray(data).nbytes, n
        info = g.info()
        assert "arch:      qwen3moe" in info and "n_layers:  2" in info and "emb_dim:   256" in info
        assert "q4_k: 6" in info and "q6_k: 1" in info and "q8_0: 9" in info
        assert "unsupported GPU quant tensors:\n  none" in info
        assert "blk.0.ffn_gate_exps.weight  dims={ 256, 256, 8 }" in info


def test_info_lists_undecodable_types(tmp_path):
    decoder, gguf, _ = _mods()
    q40 = np.zeros(18 * 4, np.uint8)  # four Q4_0 blocks (64 x 2): no decoder here (nor in math.zig:194-225)
    q3k = np.zeros(110 * 2, np.uint8)  # two Q3_K superblocks (256 x 2): decodable
    gguf.write_gguf(tmp_path / "x.gguf", {"general.architecture": "llama", "general.name": "x"},
                    [("a.weight", 2, [64, 2], q40), ("b.weight", 0, [4], np.zeros(4, np.float32)),
                     ("c.weight", 11, [256, 2], q3k)])
    with decoder.GgufFile(tmp_path / "x.gguf") as g:
        info = g.info()
        unsupported = info.split("unsupported GPU quant tensors:")[1].split("first 16 tensors:")[0]
        assert "[q4_0] a.weight  dims={ 64, 2 }" in unsupported
        assert "c.weight" not in unsupported and "q3_k: 1" in info
        assert "name:      x" in info


@pytest.mark.parametrize("mutate", ["magic", "version", "truncated", "tensor_past_end"])
def test_malformed_files_rejected(tmp_path, pkg, mutate):
    decoder, _, _ = _mods()
    b = bytearray(_reference_test_bytes())
    if mutate == "magic":
        b[0] ^= 0xFF
    elif mutate == "version":
        b[4:8] = struct.pack("<I", 4)
    elif mutate == "truncated":
        b = b[:40]
    else:
        b = b[:-40]  # the tensor's 64 bytes no longer fit
    p = tmp_path / "bad.gguf"
    p.write_bytes(bytes(b))
    with pytest.raises(pkg.LtError):
        decoder.GgufFile(p)


def test_gguf_v1_counts(tmp_path):
    """Version 1 stores the tensor and metadata counts as u32 (reader.zig:70-72)."""
    decoder, _, _ = _mods()
    s = lambda x: struct.pack("<Q", len(x)) + x.encode()  # noqa: E731
    b = struct.pack("<IIII", 0x46554747, 1, 1, 1) + s("general.architecture") + struct.pack("<I", 8) + s("v1")
    b += s("w") + struct.pack("<IQIQ", 1, 8, 0, 0)
    b += b"\0" * ((-len(b)) % 32) + b"\0" * 32
    p = tmp_path / "v1.gguf"
    p.write_bytes(b)
    with decoder.GgufFile(p) as g:
        assert g.tensors() == [("w", 0, 32)]
        assert "GGUF v1" in g.info()
