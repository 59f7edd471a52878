"""ctypes front end for the CPU checker libraries (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline / reference
legs import this module: it is the checker, never the product path.

* ``libobs_oracle.so``: the C restatement of the reference's MoE arithmetic
  (obs_oracle.c; each routine cites the reference file:line it follows).
* ``_ref/libobs_refshaders.so``: the reference's own Metal kernels
  (shaders/*.metal) compiled as C++ and strung together like
  src/forward.rs:164-232, used to pin the restatement.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_f16p = np.ctypeslib.ndpointer(np.float16, flags="C_CONTIGUOUS")


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "libobs_oracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle not built: {path} (run make -C oracle)")
        L = C.CDLL(path)
        L.orc_stream_key.restype = C.c_uint64
        L.orc_stream_key.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32]
        L.orc_stream_u64.restype = C.c_uint64
        L.orc_stream_u64.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_synth_router.argtypes = [C.c_uint64, C.c_uint32, C.c_int, C.c_int, _u32p, _u16p, _u16p]
        L.orc_synth_proj.argtypes = [C.c_uint64, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_int,
                                     _u32p, _u16p, _u16p]
        L.orc_synth_x.argtypes = [C.c_uint64, C.c_uint32, C.c_int, C.c_int, C.c_int, C.c_float, _u16p]
        L.orc_rmsnorm_row.argtypes = [_u16p, C.c_int, C.c_float, _u16p]
        L.orc_rmsnorm_tg_row.argtypes = [_u16p, C.c_void_p, C.c_int, C.c_float, _u16p]
        L.orc_rms_tg.argtypes = [_u16p, C.c_int, C.c_float]
        L.orc_rms_tg.restype = C.c_float
        L.orc_dequant4.argtypes = [_u32p, _u16p, _u16p, C.c_int, C.c_int, _f32p]
        L.orc_dequant8.argtypes = [_u32p, _u16p, _u16p, C.c_int, C.c_int, _f32p]
        L.orc_dequant4_bf16.argtypes = [_u32p, _u16p, _u16p, C.c_int, C.c_int, _u16p]
        L.orc_router_logits.restype = C.c_int
        L.orc_router_logits.argtypes = [_u32p, _u16p, _u16p, _u16p, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_topk.argtypes = [_f32p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, _i32p, _f32p]
        L.orc_dispatch.argtypes = [_i32p, C.c_int, C.c_int, C.c_int, _i32p, _i32p, _i32p, _i32p]
        L.orc_moe_ffn_combine.restype = C.c_int
        L.orc_moe_ffn_combine.argtypes = [C.c_void_p, _u16p, C.c_int, _i32p, _f32p, C.c_void_p,
                                          C.c_int, C.c_int, _u16p, C.c_void_p, C.c_void_p]
        L.orc_embed.argtypes = [_u32p, _u16p, _u16p, C.c_int, C.c_int, _i32p, C.c_int, _u16p]
        L.orc_lm_head_logits.restype = C.c_int
        L.orc_lm_head_logits.argtypes = [_u32p, _u16p, _u16p, C.c_int, C.c_int, _u16p, C.c_int, C.c_int, _f32p]
        L.orc_argmax_rows.argtypes = [_f32p, C.c_int, C.c_int, _i32p]
        L.orc_rope_table.argtypes = [C.c_double, C.c_int, C.c_int, _f32p]
        L.orc_attn_forward.restype = C.c_int
        L.orc_attn_forward.argtypes = [C.c_void_p, _u16p, C.c_int, _i32p, _i32p, C.c_float, C.c_int, _u16p]
        L.orc_moe_layer.restype = C.c_int
        L.orc_moe_layer.argtypes = [C.c_void_p, _u16p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                    C.c_int, C.c_int, _u16p, _i32p, _f32p]
        _LIB = L
    return _LIB


# ------------------------------------------------------------------ bf16 utils
def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ------------------------------------------------------------ synthetic data
@dataclass
class Layer:
    """One MoE layer in the reference's host format (MLX affine, row-major)."""
    E: int
    H: int
    I: int
    K: int
    router_w: np.ndarray
    router_s: np.ndarray
    router_b: np.ndarray
    gate_w: np.ndarray
    gate_s: np.ndarray
    gate_b: np.ndarray
    up_w: np.ndarray
    up_s: np.ndarray
    up_b: np.ndarray
    down_w: np.ndarray
    down_s: np.ndarray
    down_b: np.ndarray


def synth_router(seed, layer, E, H):
    w = np.empty((E, H // 4), np.uint32)
    s = np.empty((E, H // 64), np.uint16)
    b = np.empty((E, H // 64), np.uint16)
    lib().orc_synth_router(seed, layer, E, H, w, s, b)
    return w, s, b


def synth_proj(seed, layer, proj, E, out_f, in_f):
    w = np.empty((E, out_f, in_f // 8), np.uint32)
    s = np.empty((E, out_f, in_f // 64), np.uint16)
    b = np.empty((E, out_f, in_f // 64), np.uint16)
    lib().orc_synth_proj(seed, layer, proj, E, out_f, in_f, w, s, b)
    return w, s, b


def synth_layer(seed=0, layer=0, E=128, H=2048, I=768, K=8) -> Layer:
    rw, rs, rb = synth_router(seed, layer, E, H)
    gw, gs, gb = synth_proj(seed, layer, 0, E, I, H)
    uw, us, ub = synth_proj(seed, layer, 1, E, I, H)
    dw, ds, db = synth_proj(seed, layer, 2, E, H, I)
    return Layer(E, H, I, K, rw, rs, rb, gw, gs, gb, uw, us, ub, dw, ds, db)


def synth_x(seed, layer, T, H, row0=0, eps=1e-6):
    x = np.empty((T, H), np.uint16)
    lib().orc_synth_x(seed, layer, row0, T, H, eps, x)
    return x


def rmsnorm_layer(x, eps=1e-6):
    """The MoE stack's layer-input RMSNorm in rmsnorm.metal's threadgroup order (weight 1)."""
    x = np.ascontiguousarray(x, np.uint16)
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        lib().orc_rmsnorm_tg_row(x[t], None, x.shape[1], eps, out[t])
    return out


def rms_layer(x, eps=1e-6):
    """The fp32 rms of each row in rmsnorm.metal's reduction order."""
    x = np.ascontiguousarray(x, np.uint16)
    return np.array([lib().orc_rms_tg(x[t], x.shape[1], eps) for t in range(x.shape[0])], np.float32)


def rmsnorm(x, eps=1e-6):
    x = np.ascontiguousarray(x, np.uint16)
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        lib().orc_rmsnorm_row(x[t], x.shape[1], eps, out[t])
    return out


# -------------------------------------------------------------- the checker
def dequant4(w, s, b):
    out_f, words = w.shape[-2], w.shape[-1]
    out = np.empty((out_f, words * 8), np.float32)
    lib().orc_dequant4(np.ascontiguousarray(w), np.ascontiguousarray(s), np.ascontiguousarray(b),
                       out_f, words * 8, out)
    return out


def dequant4_bf16(w, s, b):
    """Tensor-core path weights: bf16 of the exact q*s + b, one rounding."""
    out_f, words = w.shape[-2], w.shape[-1]
    out = np.empty((out_f, words * 8), np.uint16)
    lib().orc_dequant4_bf16(np.ascontiguousarray(w), np.ascontiguousarray(s), np.ascontiguousarray(b),
                            out_f, words * 8, out)
    return out


def dequant8(w, s, b):
    out_f, words = w.shape
    out = np.empty((out_f, words * 4), np.float32)
    lib().orc_dequant8(np.ascontiguousarray(w), np.ascontiguousarray(s), np.ascontiguousarray(b),
                       out_f, words * 4, out)
    return out


def router_logits(L: Layer, x):
    T = x.shape[0]
    out = np.empty((T, L.E), np.float32)
    rc = lib().orc_router_logits(L.router_w, L.router_s, L.router_b, np.ascontiguousarray(x),
                                 T, L.H, L.E, out)
    if rc:
        raise ValueError("router_logits: hidden size must be a multiple of 2048")
    return out


def topk(logits, K, bias=None, norm=True):
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    ids = np.empty((T, K), np.int32)
    w = np.empty((T, K), np.float32)
    bias_arr = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib().orc_topk(logits, None if bias_arr is None else bias_arr.ctypes.data, T, E, K, int(norm), ids, w)
    return ids, w


def dispatch(ids, E):
    ids = np.ascontiguousarray(ids, np.int32)
    T, K = ids.shape
    counts = np.empty(E, np.int32)
    offsets = np.empty(E + 1, np.int32)
    slot_of = np.empty((T, K), np.int32)
    src = np.empty(max(T * K, 1), np.int32)
    lib().orc_dispatch(ids, T, E, K, counts, offsets, slot_of, src)
    return counts, offsets, slot_of, src[: T * K]


class _Experts(C.Structure):
    _fields_ = [("E", C.c_int), ("H", C.c_int), ("I", C.c_int), ("K", C.c_int),
                ("gate_w", C.c_void_p), ("up_w", C.c_void_p), ("down_w", C.c_void_p),
                ("gate_s", C.c_void_p), ("gate_b", C.c_void_p), ("up_s", C.c_void_p),
                ("up_b", C.c_void_p), ("down_s", C.c_void_p), ("down_b", C.c_void_p)]


class _Layer(C.Structure):
    _fields_ = [("ex", _Experts), ("router_w", C.c_void_p), ("router_s", C.c_void_p),
                ("router_b", C.c_void_p)]


def _experts_struct(L: Layer):
    return _Experts(L.E, L.H, L.I, L.K, L.gate_w.ctypes.data, L.up_w.ctypes.data,
                    L.down_w.ctypes.data, L.gate_s.ctypes.data, L.gate_b.ctypes.data,
                    L.up_s.ctypes.data, L.up_b.ctypes.data, L.down_s.ctypes.data,
                    L.down_b.ctypes.data)


def moe_ffn_combine(L: Layer, x, ids, weights, residual=None, wmode=0, nthreads=None,
                    want_h=False, want_y=False):
    """Expert FFN + rank-order combine.  Returns out (and h [T,K,I], y [T,K,H])."""
    x = np.ascontiguousarray(x, np.uint16)
    T = x.shape[0]
    nthreads = nthreads or os.cpu_count() or 1
    out = np.empty((T, L.H), np.uint16)
    h = np.empty((T, L.K, L.I), np.uint16) if want_h else None
    y = np.empty((T, L.K, L.H), np.uint16) if want_y else None
    res = None if residual is None else np.ascontiguousarray(residual, np.uint16)
    ex = _experts_struct(L)
    rc = lib().orc_moe_ffn_combine(C.byref(ex), x, T, np.ascontiguousarray(ids, np.int32),
                                   np.ascontiguousarray(weights, np.float32),
                                   None if res is None else res.ctypes.data, wmode, nthreads, out,
                                   None if h is None else h.ctypes.data,
                                   None if y is None else y.ctypes.data)
    if rc:
        raise ValueError("moe_ffn_combine: bad shapes")
    return out, h, y


def moe_layer(L: Layer, x, bias=None, residual=None, norm_topk=True, wmode=0, nthreads=None):
    """Full layer on the CPU: router -> top-k -> FFN -> combine.  (out, ids, w)."""
    x = np.ascontiguousarray(x, np.uint16)
    T = x.shape[0]
    nthreads = nthreads or os.cpu_count() or 1
    out = np.empty((T, L.H), np.uint16)
    ids = np.empty((T, L.K), np.int32)
    w = np.empty((T, L.K), np.float32)
    bias_arr = None if bias is None else np.ascontiguousarray(bias, np.float32)
    res = None if residual is None else np.ascontiguousarray(residual, np.uint16)
    ex = _Layer(_experts_struct(L), L.router_w.ctypes.data, L.router_s.ctypes.data,
                L.router_b.ctypes.data)
    rc = lib().orc_moe_layer(C.byref(ex), x, T, None if bias_arr is None else bias_arr.ctypes.data,
                             None if res is None else res.ctypes.data, int(norm_topk), wmode,
                             nthreads, out, ids, w)
    if rc:
        raise ValueError("moe_layer failed")
    return out, ids, w


def moe_stack(layers, r0, bias=None, eps=1e-6, wmode=0, nthreads=None):
    """A chain of MoE layers with a residual stream (BASELINE configs 2 and 3,
    forward.rs:419-441 without attention): x_l = RMSNorm(r_l) in rmsnorm.metal's
    order, r_{l+1} = r_l + MoE_l(x_l) (combine with the residual, rounded once)."""
    r = np.ascontiguousarray(r0, np.uint16)
    for L in layers:
        x = rmsnorm_layer(r, eps)
        r, _, _ = moe_layer(L, x, bias=bias, residual=r, wmode=wmode, nthreads=nthreads)
    return r


# ---------------------------------------------------------- the model's ends
@dataclass
class Head:
    """Embedding, final norm weight and lm_head in the MLX 4-bit layout."""
    vocab: int
    H: int
    embed_w: np.ndarray
    embed_s: np.ndarray
    embed_b: np.ndarray
    lm_w: np.ndarray
    lm_s: np.ndarray
    lm_b: np.ndarray
    norm_w: np.ndarray


def synth_head(seed=0, vocab=151936, H=2048):
    """Seeded head: the embedding and lm_head drawn like an expert projection
    ((seed, layer 1000 / 1001) streams), the final norm weight ~ 1 + U(-0.1, 0.1)."""
    ew, es, eb = synth_proj(seed, 1000, 0, 1, vocab, H)
    lw, ls, lb = synth_proj(seed, 1001, 0, 1, vocab, H)
    rng = np.random.default_rng(seed + 7)
    norm_w = f32_to_bf16((1.0 + rng.uniform(-0.1, 0.1, H)).astype(np.float32))
    return Head(vocab, H, ew[0], es[0], eb[0], lw[0], ls[0], lb[0], norm_w)


def embed(head: Head, tokens):
    tokens = np.ascontiguousarray(tokens, np.int32)
    out = np.empty((tokens.size, head.H), np.uint16)
    lib().orc_embed(head.embed_w, head.embed_s, head.embed_b, head.vocab, head.H, tokens, tokens.size, out)
    return out


def lm_head(head: Head, x, nthreads=None):
    """Final RMSNorm (model.norm) in rmsnorm.metal's order, lm_head logits in the
    canonical order, and the first maximum: (logits fp32 [T, vocab], ids [T])."""
    x = np.ascontiguousarray(x, np.uint16)
    T = x.shape[0]
    xn = np.empty_like(x)
    for t in range(T):
        lib().orc_rmsnorm_tg_row(x[t], head.norm_w.ctypes.data, head.H, 1e-6, xn[t])
    logits = np.empty((T, head.vocab), np.float32)
    rc = lib().orc_lm_head_logits(head.lm_w, head.lm_s, head.lm_b, head.vocab, head.H, xn, T,
                                  nthreads or os.cpu_count() or 1, logits)
    if rc:
        raise ValueError("lm_head: hidden size must be a multiple of 2048")
    ids = np.empty(T, np.int32)
    lib().orc_argmax_rows(logits, T, head.vocab, ids)
    return logits, ids


# ------------------------------------------------------- the attention block
@dataclass
class Attn:
    """One layer's attention weights (MLX 4-bit) and the shape of its block."""
    H: int
    nq: int
    nkv: int
    hd: int
    q_w: np.ndarray
    q_s: np.ndarray
    q_b: np.ndarray
    k_w: np.ndarray
    k_s: np.ndarray
    k_b: np.ndarray
    v_w: np.ndarray
    v_s: np.ndarray
    v_b: np.ndarray
    o_w: np.ndarray
    o_s: np.ndarray
    o_b: np.ndarray
    in_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray


def synth_attn(seed=0, layer=0, H=2048, nq=32, nkv=4, hd=128):
    """Seeded attention weights: q/k/v/o drawn like expert projections from the
    (seed, 2000 + 4*layer + i) streams, norm weights ~ 1 + U(-0.1, 0.1)."""
    rq, rk = nq * hd, nkv * hd
    qw, qs, qb = (a[0] for a in synth_proj(seed, 2000 + 4 * layer, 0, 1, rq, H))
    kw, ks, kb = (a[0] for a in synth_proj(seed, 2001 + 4 * layer, 0, 1, rk, H))
    vw, vs, vb = (a[0] for a in synth_proj(seed, 2002 + 4 * layer, 0, 1, rk, H))
    ow, os_, ob = (a[0] for a in synth_proj(seed, 2003 + 4 * layer, 0, 1, H, rq))
    rng = np.random.default_rng(seed * 1000 + layer + 3)
    nrm = lambda n: f32_to_bf16((1.0 + rng.uniform(-0.1, 0.1, n)).astype(np.float32))  # noqa: E731
    return Attn(H, nq, nkv, hd, qw, qs, qb, kw, ks, kb, vw, vs, vb, ow, os_, ob, nrm(H), nrm(hd), nrm(hd))


class _Attn(C.Structure):
    _fields_ = [("H", C.c_int), ("nq", C.c_int), ("nkv", C.c_int), ("hd", C.c_int), ("max_seq", C.c_int),
                ("n_seqs", C.c_int)] + [(n, C.c_void_p) for n in (
                    "q_w", "k_w", "v_w", "o_w", "q_s", "q_b", "k_s", "k_b", "v_s", "v_b", "o_s", "o_b",
                    "in_norm", "q_norm", "k_norm", "rope", "kc", "vc")]


class AttnState:
    """The oracle's KV caches for n_seqs sequences and its RoPE table."""

    def __init__(self, A: Attn, max_seq, n_seqs, theta=1e7):
        self.A, self.max_seq, self.n_seqs = A, max_seq, n_seqs
        self.kc = np.zeros((n_seqs, A.nkv, max_seq, A.hd), np.uint16)
        self.vc = np.zeros_like(self.kc)
        self.rope = np.empty((max_seq, A.hd // 2, 2), np.float32)
        lib().orc_rope_table(theta, A.hd, max_seq, self.rope)

    def forward(self, x, seq, pos, eps=1e-6, nthreads=None):
        A = self.A
        x = np.ascontiguousarray(x, np.uint16)
        T = x.shape[0]
        out = np.empty_like(x)
        st = _Attn(A.H, A.nq, A.nkv, A.hd, self.max_seq, self.n_seqs,
                   *[getattr(A, n).ctypes.data for n in ("q_w", "k_w", "v_w", "o_w", "q_s", "q_b", "k_s", "k_b",
                                                         "v_s", "v_b", "o_s", "o_b", "in_norm", "q_norm", "k_norm")],
                   self.rope.ctypes.data, self.kc.ctypes.data, self.vc.ctypes.data)
        rc = lib().orc_attn_forward(C.byref(st), x, T, np.ascontiguousarray(seq, np.int32),
                                    np.ascontiguousarray(pos, np.int32), eps, nthreads or os.cpu_count() or 1, out)
        if rc:
            raise ValueError("attn_forward: bad shape")
        return out


# ------------------------------------------- reference shaders (CPU build)
def ref_lib():
    """The reference's own kernels compiled for the CPU, or None if not built."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libobs_refshaders.so")
        if not os.path.exists(path):
            return None
        R = C.CDLL(path)
        R.ref_dequant_matvec_8bit.argtypes = [_u32p, _f16p, _f16p, _f16p, _f16p, C.c_int, C.c_int]
        R.ref_fused_dequant_matvec_4bit.argtypes = [_u32p, _f16p, _f16p, _f16p, _f16p, C.c_int,
                                                    C.c_int, C.c_int]
        R.ref_matmul_dequant_4bit.argtypes = [_u32p, _f16p, _f16p, _f16p, _f16p, C.c_int, C.c_int,
                                              C.c_int, C.c_int]
        R.ref_moe_routing_topk.argtypes = [_f16p, C.c_int, C.c_int, C.c_int, _i32p, _f16p]
        R.ref_ew_swiglu.argtypes = [_f16p, _f16p, _f16p, C.c_int]
        R.ref_ew_scaled_add.argtypes = [_f16p, _f16p, C.c_float, C.c_int]
        R.ref_rmsnorm.argtypes = [_f16p, _f16p, _f16p, C.c_int, C.c_int, C.c_float]
        R.ref_rope.argtypes = [_f16p, C.c_int, C.c_int, C.c_int, C.c_float]
        R.ref_attn_token.restype = C.c_int
        R.ref_attn_token.argtypes = [C.c_void_p, _f16p, _f16p, C.c_int, _u16p, C.c_int, _f16p]
        R.ref_moe_prefill.restype = C.c_int
        R.ref_moe_prefill.argtypes = [C.c_void_p, _u16p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, _f16p,
                                      _i32p, _f32p]
        _REF = R
    return _REF


def ref_route(L: Layer, x, norm=True):
    """The reference's router on the CPU, token by token as forward.rs:386-397 and
    router.rs:25-56 run it: dequant_matvec_8bit (logits rounded to f16) then
    moe_routing_topk.  Returns (logits f16 [T, E], ids [T, K], weights f16 [T, K])."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("oracle/_ref not built")
    x = np.ascontiguousarray(x, np.uint16)
    T = x.shape[0]
    s16 = bf16_to_f32(L.router_s).astype(np.float16)
    b16 = bf16_to_f32(L.router_b).astype(np.float16)
    x16 = bf16_to_f32(x).astype(np.float16)
    logits = np.empty((T, L.E), np.float16)
    ids = np.empty((T, L.K), np.int32)
    w = np.empty((T, L.K), np.float16)
    for t in range(T):
        R.ref_dequant_matvec_8bit(L.router_w, s16, b16, np.ascontiguousarray(x16[t]), logits[t], L.H, L.E)
        R.ref_moe_routing_topk(np.ascontiguousarray(logits[t]), L.E, L.K, int(norm), ids[t], w[t])
    return logits, ids, w


class _RefLayer(C.Structure):
    _fields_ = [("E", C.c_int), ("H", C.c_int), ("I", C.c_int), ("K", C.c_int),
                ("router_w", C.c_void_p), ("gate_w", C.c_void_p), ("up_w", C.c_void_p),
                ("down_w", C.c_void_p), ("router_s", C.c_void_p), ("router_b", C.c_void_p),
                ("gate_s", C.c_void_p), ("gate_b", C.c_void_p), ("up_s", C.c_void_p),
                ("up_b", C.c_void_p), ("down_s", C.c_void_p), ("down_b", C.c_void_p)]


def ref_moe_prefill(L: Layer, x, residual=None, nthreads=None, bias=None):
    """The reference's batched-prefill MoE section on the CPU: (out f16, ids, w)."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("oracle/_ref not built")
    x = np.ascontiguousarray(x, np.uint16)
    T = x.shape[0]
    nthreads = nthreads or os.cpu_count() or 1
    out = np.empty((T, L.H), np.float16)
    ids = np.empty((T, L.K), np.int32)
    w = np.empty((T, L.K), np.float32)
    st = _RefLayer(L.E, L.H, L.I, L.K, L.router_w.ctypes.data, L.gate_w.ctypes.data,
                   L.up_w.ctypes.data, L.down_w.ctypes.data, L.router_s.ctypes.data,
                   L.router_b.ctypes.data, L.gate_s.ctypes.data, L.gate_b.ctypes.data,
                   L.up_s.ctypes.data, L.up_b.ctypes.data, L.down_s.ctypes.data,
                   L.down_b.ctypes.data)
    res = None if residual is None else np.ascontiguousarray(residual, np.uint16)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    R.ref_moe_prefill(C.byref(st), x, None if res is None else res.ctypes.data, None if b is None else b.ctypes.data,
                      T, nthreads, out, ids, w)
    return out, ids, w


class _RefAttn(C.Structure):
    _fields_ = [("H", C.c_int), ("nq", C.c_int), ("nkv", C.c_int), ("hd", C.c_int), ("max_len", C.c_int),
                ("theta", C.c_float), ("eps", C.c_float)] + [(n, C.c_void_p) for n in (
                    "q_w", "k_w", "v_w", "o_w", "q_s", "q_b", "k_s", "k_b", "v_s", "v_b", "o_s", "o_b",
                    "in_norm", "q_norm", "k_norm")]


class RefAttnState:
    """The reference's attention block on the CPU (its own kernels, forward.rs:404-419),
    one decode token per call, with its f16 KV caches [n_kv][max_len][head_dim]."""

    def __init__(self, A: Attn, max_len, theta=1e7, eps=1e-6):
        if ref_lib() is None:
            raise RuntimeError("oracle/_ref not built")
        self.A, self.max_len = A, max_len
        self.kc = np.zeros((A.nkv, max_len, A.hd), np.float16)
        self.vc = np.zeros_like(self.kc)
        self._st = _RefAttn(A.H, A.nq, A.nkv, A.hd, max_len, theta, eps,
                            *[getattr(A, n).ctypes.data for n in (
                                "q_w", "k_w", "v_w", "o_w", "q_s", "q_b", "k_s", "k_b", "v_s", "v_b", "o_s", "o_b",
                                "in_norm", "q_norm", "k_norm")])

    def token(self, x_row, pos, nthreads=None):
        out = np.empty(self.A.H, np.float16)
        rc = ref_lib().ref_attn_token(C.byref(self._st), self.kc, self.vc, int(pos),
                                      np.ascontiguousarray(x_row, np.uint16), nthreads or os.cpu_count() or 1, out)
        if rc:
            raise ValueError("ref_attn_token: position out of range")
        return out


def ref_rope(x16, pos, theta=1e7):
    """rope.metal on the CPU: x16 f16 [n_heads, head_dim] rotated in place at pos."""
    x16 = np.ascontiguousarray(x16, np.float16)
    ref_lib().ref_rope(x16, x16.shape[0], x16.shape[1], int(pos), theta)
    return x16
