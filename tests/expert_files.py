"""Per-layer expert files in the reference splitter's format, for the loader tests.

tools/split_experts.py:63-75 writes layer_{il}_experts.safetensors with, for each
expert e and projection p, e{e}.{p}.weight (uint32, the packed 4-bit codes as
stored in the MLX checkpoint) and e{e}.{p}.scales / .biases cast from the
checkpoint's bf16 to float16.  This writes the same file from an oracle layer
(whose scales and biases are bf16) with the safetensors package, as the
splitter's mx.save_safetensors does."""
from __future__ import annotations

import numpy as np
from safetensors.numpy import save_file

import oracle as O

PROJS = ("gate_proj", "up_proj", "down_proj")


def layer_tensors(L, scale_dtype=np.float16):
    out = {}
    for p, (w, s, b) in zip(PROJS, ((L.gate_w, L.gate_s, L.gate_b), (L.up_w, L.up_s, L.up_b),
                                     (L.down_w, L.down_s, L.down_b))):
        for e in range(L.E):
            out[f"e{e}.{p}.weight"] = np.ascontiguousarray(w[e])
            if scale_dtype is None:  # keep bf16 bit patterns (written as BF16 below)
                out[f"e{e}.{p}.scales"] = np.ascontiguousarray(s[e])
                out[f"e{e}.{p}.biases"] = np.ascontiguousarray(b[e])
            else:  # the splitter's t.astype(mx.float16): bf16 -> f16, round to nearest
                out[f"e{e}.{p}.scales"] = O.bf16_to_f32(s[e]).astype(scale_dtype)
                out[f"e{e}.{p}.biases"] = O.bf16_to_f32(b[e]).astype(scale_dtype)
    return out


def write_layer_file(path, L, drop=None, extra=None):
    """The splitter's file for layer L; drop: a tensor name to leave out; extra:
    more tensors (a non-expert name the loader must skip)."""
    t = layer_tensors(L)
    if drop:
        t.pop(drop)
    if extra:
        t.update(extra)
    save_file(t, str(path), metadata={"format": "mlx"})
    return path
