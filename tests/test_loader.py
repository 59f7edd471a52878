"""The expert-file loader's header reader without a GPU (obs_expert_file_info):
the reference splitter's per-layer safetensors files (tools/split_experts.py:63-75,
indexed by src/disk_io.rs:36-63) are recognised, and malformed ones are refused
with a message."""
import numpy as np
import pytest

import obsmoe
import oracle as O
from expert_files import layer_tensors, write_layer_file
from safetensors.numpy import save_file


@pytest.fixture(scope="module")
def layer():
    return O.synth_layer(3, 0, E=4, H=2048, I=256, K=2)


def test_info_of_a_splitter_file(tmp_path, layer):
    p = write_layer_file(tmp_path / "layer_0_experts.safetensors", layer)
    assert obsmoe.expert_file_info(str(p)) == (4, 2048, 256)


def test_non_expert_tensors_are_skipped(tmp_path, layer):
    extra = {"lm_head.weight": np.zeros((2, 2), np.float32), "model.norm.weight": np.ones(4, np.float16)}
    p = write_layer_file(tmp_path / "x.safetensors", layer, extra=extra)
    assert obsmoe.expert_file_info(str(p)) == (4, 2048, 256)


def test_bf16_scales_are_accepted(tmp_path, layer):
    t = layer_tensors(layer, scale_dtype=None)
    # BF16 tensors: safetensors writes them from their raw bytes with dtype "BF16"
    import json
    import struct

    header, blobs, off = {}, [], 0
    for name, a in t.items():
        a = np.ascontiguousarray(a)
        dtype = "U32" if a.dtype == np.uint32 else "BF16"
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    h = json.dumps(header).encode()
    p = tmp_path / "bf16.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    assert obsmoe.expert_file_info(str(p)) == (4, 2048, 256)


@pytest.mark.parametrize("case,msg", [
    ("missing", "missing tensor of e2.up_proj"),
    ("dtype", "not F16 or BF16"),
    ("shape", "wrong shape"),
    ("garbage", "header"),
    ("empty", "no e{N}"),
    ("absent", "cannot open"),
])
def test_malformed_files_are_refused(tmp_path, layer, case, msg):
    p = tmp_path / f"{case}.safetensors"
    if case == "missing":
        write_layer_file(p, layer, drop="e2.up_proj.scales")
    elif case == "dtype":
        t = layer_tensors(layer)
        t["e1.down_proj.biases"] = t["e1.down_proj.biases"].astype(np.float32)
        save_file(t, str(p))
    elif case == "shape":
        t = layer_tensors(layer)
        t["e3.gate_proj.weight"] = t["e3.gate_proj.weight"][:, :-1].copy()
        save_file(t, str(p))
    elif case == "garbage":
        p.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{\"a\": [1, 2,,]}   ")
    elif case == "empty":
        save_file({"lm_head.weight": np.zeros(4, np.float16)}, str(p))
    with pytest.raises(obsmoe.ObsError, match=msg.replace("{", r"\{")):
        obsmoe.expert_file_info(str(p))
