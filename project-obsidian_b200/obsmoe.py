"""Python front end of libobsmoe.so (include/obs_moe.h) for the B200 MoE path.

Mirrors the reference's MoE helpers in src/forward.rs and src/router.rs by name
and argument meaning: ``gate_gpu`` (forward.rs:386-397), ``route``
(router.rs:25-56), ``dispatch`` (the grouping of forward.rs:203-216),
``expert_ffn`` (dequant/matmul_raw + swiglu, forward.rs:303-321,370-375),
``moe_forward`` (the MoE section of forward_layer / prefill_batched).  Errors
raise ``ObsError`` carrying the library's message, the way the reference's
helpers return ``Err(String)``.

Device buffers are passed as raw pointers: any object with ``data_ptr()``
(a torch CUDA tensor, used here only as device-memory plumbing) or an int.
There is no CPU fallback: if the CUDA library is missing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libobsmoe.so")

OBS_OK = 0
PATH_AUTO, PATH_DECODE, PATH_PREFILL = 0, 1, 2
_STATUS = {1: "INVALID", 2: "CUDA", 3: "NOMEM", 4: "STATE", 5: "TIMEOUT", 6: "NCCL", 7: "UNSUPPORTED"}

# every entry point include/obs_moe.h declares
EXPORTS = (
    "obs_abi_version", "obs_create", "obs_destroy", "obs_last_error", "obs_memory_bytes",
    "obs_load_layer", "obs_synth_layer", "obs_synth_activations", "obs_moe_forward",
    "obs_moe_forward_host", "obs_moe_forward_host_async", "obs_moe_host_join", "obs_gate", "obs_route", "obs_dispatch", "obs_expert_ffn",
    "obs_expert_gemm_f32", "obs_check_device", "obs_profile_enable", "obs_profile_read",
    "obs_trace_enable", "obs_decode_ffn_static", "obs_kernel_launches", "obs_ep_handle", "obs_ep_connect",
    "obs_rmsnorm", "obs_moe_stack_forward", "obs_set_wait_limit", "obs_probe_wait", "obs_struct_layout",
    "obs_load_layer_safetensors", "obs_expert_file_info", "obs_load_head", "obs_embed", "obs_lm_head",
    "obs_attn_init", "obs_load_attn", "obs_attn_forward", "obs_kv_read", "obs_debug_gemm_tiles",
    "obs_ep_set_placement", "obs_ep_get_placement", "obs_ep_plan_placement",
)
EP_HANDLE_BYTES = 64
STAGES = ("router", "topk", "dispatch", "gemm_gateup", "gemm_down", "combine", "decode_gateup", "decode_down",
          "decode_fused", "ep_send", "ep_recv", "ep_return")


class ObsError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"obs {_STATUS.get(status, status)}: {msg}")
        self.status = status


class Config(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("n_experts", C.c_int32),
                ("top_k", C.c_int32), ("group_size", C.c_int32), ("n_layers", C.c_int32),
                ("max_tokens", C.c_int32), ("norm_topk", C.c_int32),
                ("decode_max_tokens", C.c_int32), ("rms_eps", C.c_float),
                ("ep_world", C.c_int32), ("ep_rank", C.c_int32)]


class HeadWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("embed_w", "embed_s", "embed_b", "lm_w", "lm_s", "lm_b", "norm_w")]


class AttnWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "q_w", "q_s", "q_b", "k_w", "k_s", "k_b", "v_w", "v_s", "v_b", "o_w", "o_s", "o_b",
        "in_norm", "q_norm", "k_norm")]


class AttnConfig(C.Structure):
    _fields_ = [("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("max_seq", C.c_int32), ("n_seqs", C.c_int32), ("rope_theta", C.c_float)]


class LayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "router_w", "router_s", "router_b", "gate_w", "gate_s", "gate_b",
        "up_w", "up_s", "up_b", "down_w", "down_s", "down_b")]


_LIB = None


def lib() -> C.CDLL:
    """Load libobsmoe.so (built by project-obsidian_b200/build.py)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with python project-obsidian_b200/build.py")
        L = C.CDLL(LIB_PATH)
        vp, i32, i64 = C.c_void_p, C.c_int, C.c_uint64
        L.obs_abi_version.restype = i32
        L.obs_create.argtypes = [C.POINTER(Config), i32, C.POINTER(vp)]
        L.obs_destroy.argtypes = [vp]
        L.obs_last_error.restype = C.c_char_p
        L.obs_last_error.argtypes = [vp]
        L.obs_memory_bytes.argtypes = [vp, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
        L.obs_load_layer.argtypes = [vp, i32, C.POINTER(LayerWeights), i32]
        L.obs_synth_layer.argtypes = [vp, i32, i64]
        L.obs_synth_activations.argtypes = [i64, C.c_uint32, i32, i32, i32, C.c_float, vp, vp]
        L.obs_moe_forward.argtypes = [vp, i32, vp, vp, vp, i32, vp, i32, vp]
        L.obs_moe_forward_host.argtypes = [vp, i32, vp, vp, vp, i32, vp, i32, vp]
        L.obs_moe_forward_host_async.argtypes = [vp, i32, vp, vp, vp, i32, vp, i32, vp]
        L.obs_moe_host_join.argtypes = [vp, vp]
        L.obs_gate.argtypes = [vp, i32, vp, vp, i32, vp]
        L.obs_route.argtypes = [vp, vp, vp, i32, vp, vp, vp]
        L.obs_dispatch.argtypes = [vp, vp, i32, vp, vp, vp, vp]
        L.obs_expert_ffn.argtypes = [vp, i32, vp, vp, i32, i32, vp, vp]
        L.obs_expert_gemm_f32.argtypes = [vp, i32, i32, i32, vp, i32, vp, vp]
        L.obs_check_device.argtypes = [vp, vp]
        L.obs_profile_enable.argtypes = [vp, i32]
        L.obs_profile_read.argtypes = [vp, C.POINTER(C.c_float), C.POINTER(C.c_int32)]
        L.obs_trace_enable.argtypes = [vp, vp, i32]
        L.obs_kernel_launches.argtypes = [C.POINTER(C.c_uint64)]
        L.obs_ep_handle.argtypes = [vp, vp]
        L.obs_ep_connect.argtypes = [vp, vp]
        L.obs_ep_set_placement.argtypes = [vp, i32, C.POINTER(C.c_int32)]
        L.obs_ep_get_placement.argtypes = [vp, i32, C.POINTER(C.c_int32)]
        L.obs_ep_plan_placement.argtypes = [C.POINTER(C.c_int64), i32, i32, C.POINTER(C.c_int32)]
        L.obs_rmsnorm.argtypes = [vp, vp, vp, i32, vp, vp]
        L.obs_moe_stack_forward.argtypes = [vp, i32, i32, vp, i32, vp, i32, vp]
        L.obs_load_layer_safetensors.argtypes = [vp, i32, C.c_char_p, vp, vp, vp]
        L.obs_expert_file_info.argtypes = [C.c_char_p, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                           C.POINTER(C.c_int32)]
        L.obs_load_head.argtypes = [vp, i32, C.POINTER(HeadWeights), i32]
        L.obs_embed.argtypes = [vp, vp, i32, vp, vp]
        L.obs_lm_head.argtypes = [vp, vp, i32, vp, vp, vp]
        L.obs_debug_gemm_tiles.argtypes = [vp, i32, vp, i32, vp]
        L.obs_attn_init.argtypes = [vp, C.POINTER(AttnConfig)]
        L.obs_load_attn.argtypes = [vp, i32, C.POINTER(AttnWeights), i32]
        L.obs_attn_forward.argtypes = [vp, i32, vp, vp, i32, vp, vp, vp]
        L.obs_kv_read.argtypes = [vp, i32, i32, i32, i32, vp, vp, vp]
        L.obs_set_wait_limit.argtypes = [vp, i64]
        L.obs_probe_wait.argtypes = [vp, vp]
        L.obs_struct_layout.argtypes = [C.POINTER(C.c_int32), i32]
        L.obs_decode_ffn_static.argtypes = [C.POINTER(LayerWeights), i32, i32, i32, i32, vp, vp, vp, vp, i32, vp, vp]
        for name in EXPORTS:
            if name not in ("obs_last_error", "obs_abi_version"):
                getattr(L, name).restype = i32
        _LIB = L
    return _LIB


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):  # numpy array (host memory)
        return x.ctypes.data
    raise TypeError(f"cannot take a pointer of {type(x)}")


def _stream(s) -> int | None:
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream  # torch.cuda.Stream


@dataclass
class MoeShape:
    hidden: int = 2048
    inter: int = 768
    n_experts: int = 128
    top_k: int = 8
    n_layers: int = 1
    max_tokens: int = 512
    norm_topk: bool = True
    decode_max_tokens: int = 0   # <= 0: the library's default
    rms_eps: float = 1e-6
    ep_world: int = 1    # expert parallelism: ranks sharing the experts
    ep_rank: int = 0


class MoeContext:
    """One GPU's HBM-resident MoE layers (obs_create ... obs_destroy)."""

    def __init__(self, shape: MoeShape, device: int = 0):
        self.shape = shape
        cfg = Config(shape.hidden, shape.inter, shape.n_experts, shape.top_k, 64, shape.n_layers,
                     shape.max_tokens, int(shape.norm_topk), shape.decode_max_tokens, shape.rms_eps,
                     shape.ep_world, shape.ep_rank)
        h = C.c_void_p()
        rc = lib().obs_create(C.byref(cfg), device, C.byref(h))
        if rc != OBS_OK:
            raise ObsError(rc, lib().obs_last_error(None).decode())
        self._h = h
        self.device = device

    # -- plumbing
    def _chk(self, rc: int):
        if rc != OBS_OK:
            raise ObsError(rc, lib().obs_last_error(self._h).decode())

    def close(self):
        if getattr(self, "_h", None):
            lib().obs_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def memory_bytes(self):
        w, s = C.c_size_t(), C.c_size_t()
        self._chk(lib().obs_memory_bytes(self._h, C.byref(w), C.byref(s)))
        return w.value, s.value

    # -- weights
    def load_layer(self, layer: int, w, on_device: bool = False):
        """Copy one layer in the reference format (attributes router_w ... down_b)."""
        lw = LayerWeights(*[_ptr(getattr(w, n)) for n, _ in LayerWeights._fields_])
        self._chk(lib().obs_load_layer(self._h, layer, C.byref(lw), int(on_device)))

    def load_layer_file(self, layer: int, path: str, router_w, router_s, router_b):
        """One layer from the reference splitter's safetensors file (experts) plus the router
        arrays (host numpy arrays in the MLX layout)."""
        self._chk(lib().obs_load_layer_safetensors(self._h, layer, os.fsencode(path), _ptr(router_w), _ptr(router_s),
                                                   _ptr(router_b)))

    def load_head(self, vocab: int, w, on_device: bool = False):
        """The embedding, final norm and lm_head (attributes embed_w ... norm_w)."""
        hw = HeadWeights(*[_ptr(getattr(w, n)) for n, _ in HeadWeights._fields_])
        self._chk(lib().obs_load_head(self._h, vocab, C.byref(hw), int(on_device)))

    def embed(self, tokens, T, x, stream=None):
        self._chk(lib().obs_embed(self._h, _ptr(tokens), T, _ptr(x), _stream(stream)))

    def lm_head(self, x, T, ids, logits=None, stream=None):
        """RMSNorm(model.norm) -> lm_head -> greedy ids (first maximum); logits optional."""
        self._chk(lib().obs_lm_head(self._h, _ptr(x), T, _ptr(ids), _ptr(logits), _stream(stream)))

    # -- the attention block
    def attn_init(self, n_heads=32, n_kv_heads=4, head_dim=128, max_seq=4096, n_seqs=1, rope_theta=1e7):
        ac = AttnConfig(n_heads, n_kv_heads, head_dim, max_seq, n_seqs, rope_theta)
        self._chk(lib().obs_attn_init(self._h, C.byref(ac)))

    def load_attn(self, layer: int, w, on_device: bool = False):
        """One layer's attention weights (attributes q_w ... k_norm, MLX 4-bit layout)."""
        aw = AttnWeights(*[_ptr(getattr(w, n)) for n, _ in AttnWeights._fields_])
        self._chk(lib().obs_load_attn(self._h, layer, C.byref(aw), int(on_device)))

    def attn_forward(self, layer, x, out, T, seq, pos, stream=None):
        """out = x + attention(x) for T tokens of sequences seq[t] at positions pos[t]; appends K/V."""
        self._chk(lib().obs_attn_forward(self._h, layer, _ptr(x), _ptr(out), T, _ptr(seq), _ptr(pos),
                                         _stream(stream)))

    def kv_read(self, layer, seq, pos0, n, k=None, v=None, stream=None):
        self._chk(lib().obs_kv_read(self._h, layer, seq, pos0, n, _ptr(k), _ptr(v), _stream(stream)))

    def synth_layer(self, layer: int, seed: int = 0):
        self._chk(lib().obs_synth_layer(self._h, layer, seed))

    # -- the reference helpers
    def gate_gpu(self, layer, x, logits, T, stream=None):
        self._chk(lib().obs_gate(self._h, layer, _ptr(x), _ptr(logits), T, _stream(stream)))

    def route(self, logits, T, ids, weights, bias=None, stream=None):
        self._chk(lib().obs_route(self._h, _ptr(logits), _ptr(bias), T, _ptr(ids), _ptr(weights),
                                  _stream(stream)))

    def dispatch(self, ids, T, counts=None, seg=None, slot_of=None, stream=None):
        self._chk(lib().obs_dispatch(self._h, _ptr(ids), T, _ptr(counts), _ptr(seg), _ptr(slot_of),
                                     _stream(stream)))

    def expert_ffn(self, layer, x, ids, T, y, path=PATH_PREFILL, stream=None):
        self._chk(lib().obs_expert_ffn(self._h, layer, _ptr(x), _ptr(ids), T, path, _ptr(y),
                                       _stream(stream)))

    def matmul_raw_f32(self, layer, proj, expert, x, n, y, stream=None):
        """One expert projection on the tcgen05 GEMM, fp32 out (matmul_dequant_4bit)."""
        self._chk(lib().obs_expert_gemm_f32(self._h, layer, proj, expert, _ptr(x), n, _ptr(y),
                                            _stream(stream)))

    # -- expert parallelism
    def ep_handle(self) -> bytes:
        """This rank's buffer handle (obs_ep_handle), to be sent to the other ranks."""
        buf = (C.c_uint8 * EP_HANDLE_BYTES)()
        self._chk(lib().obs_ep_handle(self._h, buf))
        return bytes(buf)

    def ep_connect(self, handles):
        """Open every rank's buffer (obs_ep_connect); handles in rank order."""
        blob = b"".join(handles)
        assert len(blob) == EP_HANDLE_BYTES * self.shape.ep_world
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        self._chk(lib().obs_ep_connect(self._h, buf))

    def ep_set_placement(self, layer, experts):
        """Which GPU holds which expert (obs_ep_set_placement): experts[g*E/G + l] is GPU g's local
        expert l; layer = -1 for every layer.  Changed layers must be loaded again."""
        arr = (C.c_int32 * self.shape.n_experts)(*[int(e) for e in experts])
        self._chk(lib().obs_ep_set_placement(self._h, layer, arr))

    def ep_get_placement(self, layer) -> list:
        arr = (C.c_int32 * self.shape.n_experts)()
        self._chk(lib().obs_ep_get_placement(self._h, layer, arr))
        return list(arr)

    def moe_forward(self, layer, x, out, T, residual=None, bias=None, path=PATH_AUTO, stream=None):
        self._chk(lib().obs_moe_forward(self._h, layer, _ptr(x), _ptr(out), _ptr(residual), T,
                                        _ptr(bias), path, _stream(stream)))

    def rmsnorm(self, x, out, T, weight=None, stream=None):
        self._chk(lib().obs_rmsnorm(self._h, _ptr(x), _ptr(weight), T, _ptr(out), _stream(stream)))

    def moe_stack_forward(self, layer0, n_layers, resid, T, bias=None, path=PATH_AUTO, stream=None):
        """resid <- n_layers of (r + MoE_l(RMSNorm(r))), in place."""
        self._chk(lib().obs_moe_stack_forward(self._h, layer0, n_layers, _ptr(resid), T, _ptr(bias), path,
                                              _stream(stream)))

    def moe_forward_host(self, layer, x_host, out_host, T, residual_host=None, bias_host=None,
                         path=PATH_AUTO, stream=None):
        self._chk(lib().obs_moe_forward_host(self._h, layer, _ptr(x_host), _ptr(out_host),
                                             _ptr(residual_host), T, _ptr(bias_host), path,
                                             _stream(stream)))

    def moe_forward_host_async(self, layer, x_host, out_host, T, residual_host=None, bias_host=None,
                               path=PATH_AUTO, stream=None):
        """moe_forward_host without the wait: copies in and out on internal streams, two staging
        slots, so successive calls overlap (host_join, then synchronise, before reading out_host)."""
        self._chk(lib().obs_moe_forward_host_async(self._h, layer, _ptr(x_host), _ptr(out_host),
                                                   _ptr(residual_host), T, _ptr(bias_host), path,
                                                   _stream(stream)))

    def host_join(self, stream=None):
        """Make `stream` wait for every output copy moe_forward_host_async has issued."""
        self._chk(lib().obs_moe_host_join(self._h, _stream(stream)))

    def profile(self, enable: bool):
        self._chk(lib().obs_profile_enable(self._h, int(enable)))

    def profile_read(self) -> dict:
        """{stage: (total ms, launches)} since the last read (event times on the caller's stream)."""
        ms = (C.c_float * len(STAGES))()
        n = (C.c_int32 * len(STAGES))()
        self._chk(lib().obs_profile_read(self._h, ms, n))
        return {name: (ms[i], n[i]) for i, name in enumerate(STAGES)}

    def trace(self, buf, n_steps: int):
        """Record the gate/up GEMM pipeline timeline of CTA 0 into buf (uint64 [8, n_steps])."""
        self._chk(lib().obs_trace_enable(self._h, _ptr(buf), n_steps if buf is not None else 0))

    def debug_gemm_tiles(self, layer, tiles, stream=None):
        """Test hook: the gate/up GEMM over a given tile list (numpy int32 [n][4])."""
        import numpy as np

        t = np.ascontiguousarray(tiles, dtype=np.int32).reshape(-1, 4)
        self._chk(lib().obs_debug_gemm_tiles(self._h, layer, t.ctypes.data, len(t), _stream(stream)))

    def check_device(self, stream=None):
        self._chk(lib().obs_check_device(self._h, _stream(stream)))

    def set_wait_limit(self, limit_ns: int):
        """Limit of every bounded device-side wait (0: the default 2 s)."""
        self._chk(lib().obs_set_wait_limit(self._h, limit_ns))

    def probe_wait(self, stream=None):
        """One bounded device wait on a stamp nothing writes: it runs out after the wait limit."""
        self._chk(lib().obs_probe_wait(self._h, _stream(stream)))


def decode_ffn_static(w, n_experts, hidden, inter, top_k, x, ids, weights, T, out, residual=None, stream=None):
    """obs_decode_ffn_static: the decode FFN + combine with no context and no
    device allocation (scratch is a fixed array inside the library).  ``w``
    holds device buffers of the expert weights in the reference (MLX) layout."""
    lw = LayerWeights(None, None, None, *[_ptr(getattr(w, n)) for n, _ in LayerWeights._fields_[3:]])
    rc = lib().obs_decode_ffn_static(C.byref(lw), n_experts, hidden, inter, top_k, _ptr(x), _ptr(ids),
                                     _ptr(weights), _ptr(residual), T, _ptr(out), _stream(stream))
    if rc != OBS_OK:
        raise ObsError(rc, lib().obs_last_error(None).decode())


def expert_file_info(path: str) -> tuple[int, int, int]:
    """(n_experts, hidden, inter) of a splitter expert file, read from its header alone."""
    e, h, i = C.c_int32(), C.c_int32(), C.c_int32()
    rc = lib().obs_expert_file_info(os.fsencode(path), C.byref(e), C.byref(h), C.byref(i))
    if rc != OBS_OK:
        raise ObsError(rc, lib().obs_last_error(None).decode())
    return e.value, h.value, i.value


def plan_placement(load, world: int) -> list:
    """A balanced expert placement from per-expert loads (obs_ep_plan_placement; host only)."""
    E = len(load)
    lo = (C.c_int64 * E)(*[int(v) for v in load])
    out = (C.c_int32 * E)()
    rc = lib().obs_ep_plan_placement(lo, E, world, out)
    if rc != 0:
        raise ObsError(rc, "obs_ep_plan_placement: bad arguments")
    return list(out)


def struct_layout() -> list[int]:
    """sizeof and field offsets of obs_config and obs_layer_weights, as the library was compiled."""
    n = lib().obs_struct_layout(None, 0)
    buf = (C.c_int32 * n)()
    lib().obs_struct_layout(buf, n)
    return list(buf)


def kernel_launches() -> int:
    """Kernel launches the library has issued in this process (all contexts)."""
    n = C.c_uint64(0)
    rc = lib().obs_kernel_launches(C.byref(n))
    if rc != OBS_OK:
        raise ObsError(rc, "kernel_launches")
    return int(n.value)


def synth_activations(seed, layer, row0, T, H, x, eps=1e-6, stream=None):
    rc = lib().obs_synth_activations(seed, layer, row0, T, H, eps, _ptr(x), _stream(stream))
    if rc != OBS_OK:
        raise ObsError(rc, "synth_activations")
