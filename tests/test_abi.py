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
