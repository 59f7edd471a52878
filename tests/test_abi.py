"""The C ABI library without a GPU: it loads, exports every entry point that
include/obs_moe.h declares, and rejects bad configurations with a message."""
import ctypes as C
import os
import re

import pytest

import obsmoe

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_entry_points():
    src = open(os.path.join(ROOT, "include", "obs_moe.h")).read()
    return set(re.findall(r"^(?:int|const char\*)\s+(obs_\w+)\(", src, flags=re.M))


def test_header_and_binding_agree():
    assert header_entry_points() == set(obsmoe.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = obsmoe.lib()
    for name in header_entry_points():
        assert hasattr(lib, name), name
    assert lib.obs_abi_version() == 1


def test_graft_entry_builds_everything():
    assert os.path.exists(obsmoe.LIB_PATH)
    assert os.path.exists(os.path.join(ROOT, "oracle", "libobs_oracle.so"))


@pytest.mark.parametrize("field,value,msg", [
    ("group_size", 32, "group_size"),
    ("hidden", 1024, "hidden"),
    ("inter", 100, "inter"),
    ("n_experts", 300, "n_experts"),
    ("top_k", 0, "top_k"),
    ("max_tokens", 0, "max_tokens"),
])
def test_create_rejects_bad_config(field, value, msg):
    s = obsmoe.MoeShape()
    cfg = obsmoe.Config(s.hidden, s.inter, s.n_experts, s.top_k, 64, 1, 16, 1, 4, 1e-6)
    setattr(cfg, field, value)
    h = C.c_void_p()
    rc = obsmoe.lib().obs_create(C.byref(cfg), 0, C.byref(h))
    assert rc == 1 and not h.value
    assert msg in obsmoe.lib().obs_last_error(None).decode()


def test_null_context_is_an_error():
    lib = obsmoe.lib()
    assert lib.obs_moe_forward(None, 0, None, None, None, 1, None, 0, None) == 1
    assert lib.obs_destroy(None) == 0


# ------------------------------------------------------------ struct layouts
RUST_TYPES = {"i32": (4, 4), "u32": (4, 4), "f32": (4, 4), "u64": (8, 8), "usize": (8, 8)}


def rust_block():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    return text[text.index("```rust"):text.index("```", text.index("```rust") + 7)]


def rust_struct_layout(name):
    """repr(C) layout of a struct of the INTEGRATION.md Rust binding: (size, [(field, offset)])."""
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, rust_block(), flags=re.S).group(1)
    fields = re.findall(r"pub (\w+): ([^,]+),", body)
    off, align_max, out = 0, 1, []
    for fname, ty in fields:
        ty = ty.strip()
        size, align = (8, 8) if ty.startswith("*") else RUST_TYPES[ty]
        off = (off + align - 1) // align * align
        out.append((fname, off))
        off += size
        align_max = max(align_max, align)
    return (off + align_max - 1) // align_max * align_max, out


def header_struct_fields(name):
    src = open(os.path.join(ROOT, "include", "obs_moe.h")).read()
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), src, flags=re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    return re.findall(r"(\w+)\s*;", body.replace(",", ";"))


def test_struct_layout_of_library_ctypes_and_rust_agree():
    v = obsmoe.struct_layout()
    assert len(v) == 57
    cfg_fields = header_struct_fields("obs_config")
    lw_fields = header_struct_fields("obs_layer_weights")
    hw_fields = header_struct_fields("obs_head_weights")
    assert len(cfg_fields) == 12 and len(lw_fields) == 12 and len(hw_fields) == 7
    # the library as compiled
    lib_cfg = (v[0], list(zip(cfg_fields, v[1:13])))
    lib_lw = (v[13], list(zip(lw_fields, v[14:26])))
    lib_hw = (v[26], list(zip(hw_fields, v[27:34])))
    ct_hw = (C.sizeof(obsmoe.HeadWeights),
             [(f, getattr(obsmoe.HeadWeights, f).offset) for f, _ in obsmoe.HeadWeights._fields_])
    assert ct_hw == lib_hw
    assert rust_struct_layout("ObsHeadWeights") == lib_hw
    # the ctypes binding
    ct_cfg = (C.sizeof(obsmoe.Config), [(f, getattr(obsmoe.Config, f).offset) for f, _ in obsmoe.Config._fields_])
    ct_lw = (C.sizeof(obsmoe.LayerWeights),
             [(f, getattr(obsmoe.LayerWeights, f).offset) for f, _ in obsmoe.LayerWeights._fields_])
    assert ct_cfg == lib_cfg
    assert ct_lw == lib_lw
    # the Rust binding a maintainer of the reference would add
    assert rust_struct_layout("ObsConfig") == lib_cfg
    assert rust_struct_layout("ObsLayerWeights") == lib_lw
    # the attention structs
    aw_fields = header_struct_fields("obs_attn_weights")
    ac_fields = header_struct_fields("obs_attn_config")
    assert len(aw_fields) == 15 and len(ac_fields) == 6
    lib_aw = (v[34], list(zip(aw_fields, v[35:50])))
    lib_ac = (v[50], list(zip(ac_fields, v[51:57])))
    for ct, lib_s, rust in ((obsmoe.AttnWeights, lib_aw, "ObsAttnWeights"), (obsmoe.AttnConfig, lib_ac, "ObsAttnConfig")):
        assert (C.sizeof(ct), [(f, getattr(ct, f).offset) for f, _ in ct._fields_]) == lib_s
        assert rust_struct_layout(rust) == lib_s


def test_rust_binding_declares_every_export():
    declared = set(re.findall(r"pub fn (obs_\w+)\(", rust_block()))
    assert declared == header_entry_points()
