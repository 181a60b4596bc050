"""A small .safetensors writer for the tests (the format: 8-byte little-endian
header length, a JSON header of {name: {dtype, shape, data_offsets}} plus
"__metadata__", padded with spaces to 8 bytes, then the tensor bytes)."""
import json
import struct

import numpy as np

_DT = {np.dtype(np.float32): "F32", np.dtype(np.int8): "I8", np.dtype(np.int32): "I32", np.dtype(np.float16): "F16"}


def write(path, tensors, metadata=None):
    """tensors: {name: ndarray, or ("BF16", uint16 bit array)}."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        if isinstance(a, tuple):
            dt, arr = a
        else:
            arr = np.ascontiguousarray(a)
            dt = _DT[arr.dtype]
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def llama_names(cfg, l):
    p = f"model.layers.{l}."
    return {"attn_norm": p + "input_layernorm.weight", "wq": p + "self_attn.q_proj.weight",
            "wk": p + "self_attn.k_proj.weight", "wv": p + "self_attn.v_proj.weight", "wo": p + "self_attn.o_proj.weight",
            "mlp_norm": p + "post_attention_layernorm.weight", "w_gate": p + "mlp.gate_proj.weight",
            "w_up": p + "mlp.up_proj.weight", "w_down": p + "mlp.down_proj.weight"}
