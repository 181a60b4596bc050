"""The library's safetensors reader (host code: no GPU needed)."""
import json
import os

import numpy as np
import pytest

import oracle
import st_writer


def _st():
    from teenygrad_b200.checkpoint import SafeTensors
    return SafeTensors


def test_safetensors_read_back(tmp_path):
    r = np.random.default_rng(0)
    a = r.standard_normal((2, 3)).astype(np.float32)
    b = r.standard_normal(5).astype(np.float32)
    c = r.integers(-127, 128, (3, 2)).astype(np.int8)
    d = np.array([7, -9], np.int32)
    h = np.ones((2, 2), np.float16)
    qc = {"quant_method": "compressed-tensors", "format": "int-quantized",
          "config_groups": {"group_0": {"weights": {"num_bits": 8, "type": "int", "symmetric": True,
                                                    "strategy": "channel", "axis": 0}, "targets": ["Linear"]}},
          "ignore": ["n \"quoted\"\\path"]}
    path = os.path.join(tmp_path, "t.safetensors")
    st_writer.write(path, {"a": a, "b": ("BF16", oracle.bf16_bits(b)), "c.weight": c, "c.weight_scale": b[:3],
                           "d": d, "h": h}, {"quantization_config": json.dumps(qc), "note": "tab\there é"})
    with _st()(path) as st:
        assert st.names() == ["a", "b", "c.weight", "c.weight_scale", "d", "h"]
        assert st.info("a") == (0, (2, 3), 24)
        assert st.info("b") == (1, (5,), 10)
        assert st.info("h")[0] == -1                      # F16: listed, not a library dtype
        np.testing.assert_array_equal(st.numpy("a"), a)
        np.testing.assert_array_equal(oracle.bf16_to_f32(st.numpy("b")), oracle.round_bf16(b))
        np.testing.assert_array_equal(st.numpy("c.weight"), c)
        np.testing.assert_array_equal(st.numpy("d"), d)
        assert st.quantization_config() == qc
        assert st.metadata("note") == "tab\there é"
        assert st.metadata("missing") is None


@pytest.mark.parametrize("corrupt", ["header_len", "offsets", "size"])
def test_safetensors_rejects_corrupt_files(tmp_path, corrupt):
    from teenygrad_b200 import TeenyError
    path = os.path.join(tmp_path, "bad.safetensors")
    a = np.zeros((4, 4), np.float32)
    st_writer.write(path, {"a": a})
    raw = bytearray(open(path, "rb").read())
    if corrupt == "header_len":
        raw[0:8] = (len(raw) + 100).to_bytes(8, "little")
    else:
        n = int.from_bytes(raw[0:8], "little")
        h = json.loads(raw[8:8 + n])
        if corrupt == "offsets":
            h["a"]["data_offsets"] = [0, 10 ** 6]
        else:
            h["a"]["shape"] = [4, 5]
        hb = json.dumps(h).encode()
        hb += b" " * ((8 - len(hb) % 8) % 8)
        raw = bytearray(len(hb).to_bytes(8, "little")) + hb + raw[8 + n:]
    open(path, "wb").write(bytes(raw))
    with pytest.raises(TeenyError):
        _st()(path)
