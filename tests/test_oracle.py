"""The C oracle, pinned: against the golden outputs of the reference's own
kernels (tests/golden, made by make_golden.py from shaders/*.metal compiled
for the CPU), against an independent numpy restatement of the reference's
nibble unpack (validate_dequant.py:24-30), and on hand-built known answers."""
import hashlib

import numpy as np
import pytest

import oracle as O


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def f16_of_bf16(a):
    return O.bf16_to_f32(a).astype(np.float16)


# ---------------------------------------------------------------- dequant
def numpy_unpack4(W, S, B):
    """validate_dequant.py:24-30: nibble j of word = (w >> 4j) & 0xF."""
    out_f = W.shape[0]
    nib = np.stack([(W >> (4 * j)) & 0xF for j in range(8)], -1).reshape(out_f, -1).astype(np.float32)
    s = np.repeat(O.bf16_to_f32(S), 64, axis=1)
    b = np.repeat(O.bf16_to_f32(B), 64, axis=1)
    return nib * s + b   # q*s is exact in fp32 for 4-bit codes and bf16 scales


def test_dequant4_bit_exact_vs_numpy_replica():
    w, s, b = O.synth_proj(1, 0, 0, 2, 128, 2048)
    for e in range(2):
        ref = numpy_unpack4(w[e], s[e], b[e])
        got = O.dequant4(w[e], s[e], b[e])
        assert np.array_equal(ref.view(np.uint32), got.view(np.uint32))


def test_dequant8_bit_exact_vs_byte_order():
    w, s, b = O.synth_router(1, 0, 16, 2048)
    codes = w.view(np.uint8).reshape(16, 2048).astype(np.float32)  # byte i = column i (little endian)
    ref = codes * np.repeat(O.bf16_to_f32(s), 64, 1) + np.repeat(O.bf16_to_f32(b), 64, 1)
    assert np.array_equal(ref.view(np.uint32), O.dequant8(w, s, b).view(np.uint32))


def test_nibble_order_single_word_kat():
    # word 0x76543210: nibble j holds j -> columns 0..7 dequantise to j*s + b
    w = np.zeros((1, 8), np.uint32)
    w[0, 0] = 0x76543210
    w[0, 1] = 0xFFFFFFFF  # all-15 codes
    s = np.full((1, 1), O.f32_to_bf16(np.float32(0.5)), np.uint16)
    b = np.full((1, 1), O.f32_to_bf16(np.float32(-1.0)), np.uint16)
    d = O.dequant4(w, s, b)[0]
    assert list(d[:8]) == [j * 0.5 - 1.0 for j in range(8)]
    assert list(d[8:16]) == [15 * 0.5 - 1.0] * 8
    assert np.all(d[16:] == -1.0)


# --------------------------------------------------- golden (reference kernels)
def test_golden_matvec4(golden):
    g = golden("matvec4")
    w, s, b = O.synth_proj(int(g["seed"]), 0, 0, 1, 256, 2048)
    x = O.synth_x(int(g["seed"]), 0, 3, 2048)
    assert sha(w[0], s[0], b[0], x) == str(g["input_sha"])
    # the reference's own invariant: the batched GEMM equals the per-token matvec bit for bit
    assert np.array_equal(g["matvec"].view(np.uint16), g["matmul"].view(np.uint16))
    W = O.dequant4(w[0], s[0], b[0])
    xf = f16_of_bf16(x).astype(np.float32)  # the reference computes on f16 activations
    mine = xf @ W.T
    ref = g["matvec"].astype(np.float32)
    assert np.abs(mine - ref).max() <= 2e-3 * np.abs(ref).max()


def test_golden_router_logits(golden):
    g = golden("matvec8")
    w, s, b = O.synth_router(int(g["seed"]), int(g["layer"]), 128, 2048)
    x = O.synth_x(int(g["seed"]), int(g["layer"]), 2, 2048)
    assert sha(w, s, b, x) == str(g["input_sha"])
    L = O.Layer(128, 2048, 768, 8, w, s, b, *([None] * 9))
    mine = O.router_logits(L, x)
    ref = g["logits"].astype(np.float32)
    # reference rounds logits to f16 (dequant_matvec_8bit.metal:30)
    assert np.abs(mine - ref).max() <= 2.0 ** -9 * np.abs(ref).max() + 1e-3
    assert np.array_equal(np.argsort(-ref, axis=1, kind="stable")[:, :3],
                          np.argsort(-mine, axis=1, kind="stable")[:, :3])


def test_golden_topk_ties(golden):
    g = golden("topk")
    ids, w = O.topk(g["logits"].astype(np.float32), 8)
    assert np.array_equal(ids, g["ids"])
    assert np.allclose(w, g["weights"].astype(np.float32), atol=1e-3)
    assert list(g["ids"][6]) == list(range(8))         # all-equal logits: lowest indices
    assert list(g["ids"][7][:4]) == [3, 40, 77, 100]   # four-way tie broken by index


def test_golden_moe_prefill(golden):
    g = golden("moe_prefill")
    L = O.synth_layer(int(g["seed"]), 0, E=16, H=2048, I=256, K=4)
    x = O.synth_x(int(g["seed"]), 0, 8, 2048)
    assert sha(L.router_w, L.router_s, L.router_b, L.gate_w, L.gate_s, L.gate_b, L.up_w, L.up_s, L.up_b,
               L.down_w, L.down_s, L.down_b, x) == str(g["input_sha"])
    out, ids, w = O.moe_layer(L, x, nthreads=4)
    assert all(set(a) == set(b) for a, b in zip(ids, g["ids"]))
    ref = g["out"].astype(np.float32)
    mine = O.bf16_to_f32(out)
    assert np.abs(mine - ref).max() <= 1e-2 * np.abs(ref).max()


# ----------------------------------------------------------- known answers
def test_topk_lowest_index_wins_and_renormalises():
    logits = np.zeros((1, 16), np.float32)
    logits[0, [5, 9, 2]] = 1.0
    ids, w = O.topk(logits, 4)
    assert list(ids[0]) == [2, 5, 9, 0]
    assert abs(w.sum() - 1.0) < 1e-6
    ids_b, _ = O.topk(logits, 4, bias=np.arange(16, dtype=np.float32) * 0.0 + np.eye(16, dtype=np.float32)[15] * 5)
    assert ids_b[0, 0] == 15


def test_dispatch_empty_and_hot_expert():
    T, K, E = 12, 3, 8
    ids = np.array([[0, 1, 2]] * T, np.int32)  # experts 3..7 empty; 0,1,2 get every token
    counts, offsets, slot_of, src = O.dispatch(ids, E)
    assert list(counts) == [T, T, T, 0, 0, 0, 0, 0]
    assert list(offsets) == [0, T, 2 * T] + [3 * T] * 6
    assert list(src[:T]) == list(range(T))            # token order inside a segment
    assert slot_of[5, 1] == T + 5


def test_router_order_is_the_pairwise_tree():
    # the canonical order: 32 lane chains over 64-column groups, then the adjacent pairwise tree
    w, s, b = O.synth_router(4, 0, 4, 2048)
    x = O.synth_x(4, 0, 1, 2048)
    L = O.Layer(4, 2048, 768, 2, w, s, b, *([None] * 9))
    got = O.router_logits(L, x)[0]
    W = O.dequant8(w, s, b)
    xf = O.bf16_to_f32(x[0])
    for e in range(4):
        lanes = []
        for g in range(32):
            acc = np.float32(0)
            for j in range(64):
                c = g * 64 + j
                acc = np.float32(np.fma(W[e, c], xf[c], acc)) if hasattr(np, "fma") else \
                    np.float32(float(W[e, c]) * float(xf[c]) + float(acc))
            lanes.append(acc)
        while len(lanes) > 1:
            lanes = [np.float32(lanes[i] + lanes[i + 1]) for i in range(0, len(lanes), 2)]
        assert abs(float(lanes[0]) - float(got[e])) <= 1e-6 * max(1.0, abs(float(got[e])))


@pytest.mark.parametrize("wmode", [0, 1])
def test_ffn_combine_linear_in_weights(wmode):
    # combine is linear in the routing weights: doubling w doubles out (within bf16 rounding)
    L = O.synth_layer(9, 0, E=8, H=2048, I=128, K=2)
    x = O.synth_x(9, 0, 3, 2048)
    ids = np.array([[0, 3], [3, 7], [1, 0]], np.int32)
    w = np.array([[0.6, 0.4], [0.3, 0.7], [0.5, 0.5]], np.float32)
    o1, _, y = O.moe_ffn_combine(L, x, ids, w, wmode=wmode, want_y=True)
    o2, _, _ = O.moe_ffn_combine(L, x, ids, 2 * w, wmode=wmode)
    a, b = O.bf16_to_f32(o1), O.bf16_to_f32(o2)
    assert np.abs(2 * a - b).max() <= 2 ** -7 * np.abs(b).max()
    # y rows are per (token, rank); combine = sum_k w_k y_k
    yf = O.bf16_to_f32(y)
    ref = (w[:, :, None] * yf).sum(1)
    assert np.abs(ref - a).max() <= 2 ** -7 * np.abs(ref).max()


def test_synth_distributions():
    L = O.synth_layer(0, 0, E=4, H=2048, I=128, K=2)
    s = O.bf16_to_f32(L.gate_s)
    assert 0.002 * (1 - 2 ** -8) <= s.min() and s.max() <= 0.02 * (1 + 2 ** -8)  # bf16 rounding
    b = O.bf16_to_f32(L.gate_b)
    assert np.abs(b + 8 * s).max() < 0.01                  # b = -8 s + N(0, 1e-3)
    rs, rb = O.bf16_to_f32(L.router_s), O.bf16_to_f32(L.router_b)
    assert np.array_equal(rb, -128 * rs)
    nib = np.stack([(L.gate_w >> (4 * j)) & 0xF for j in range(8)], -1)
    assert abs(nib.mean() - 7.5) < 0.05
    x = O.bf16_to_f32(O.synth_x(0, 0, 16, 2048))
    rms = np.sqrt((x * x).mean(1))
    assert np.allclose(rms, 1.0, atol=1e-2)


def test_oracle_matches_reference_shaders_live():
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built")
    L = O.synth_layer(21, 1, E=16, H=2048, I=256, K=4)
    x = O.synth_x(21, 1, 16, 2048)
    res = O.synth_x(22, 1, 16, 2048)
    out, ids, _ = O.moe_layer(L, x, residual=res, nthreads=4)
    rout, rids, _ = O.ref_moe_prefill(L, x, residual=res, nthreads=4)
    assert all(set(a) == set(b) for a, b in zip(ids, rids))
    ref = rout.astype(np.float32)
    assert np.abs(O.bf16_to_f32(out) - ref).max() <= 1e-2 * np.abs(ref).max()


def test_dequant4_bf16_single_rounding():
    # for these distributions q*s + b is exact in fp32, so one rounding equals fp32-then-bf16
    w, s, b = O.synth_proj(2, 0, 1, 1, 128, 2048)
    a = O.dequant4_bf16(w[0], s[0], b[0])
    c = O.f32_to_bf16(O.dequant4(w[0], s[0], b[0]))
    assert np.array_equal(a, c)
    # a tie case: 1 + 2^-8 lies halfway between two bf16 values -> even mantissa (1.0)
    w1 = np.zeros((1, 8), np.uint32)
    w1[0, 0] = 1                                  # code 1 in column 0
    s1 = np.array([[O.f32_to_bf16(np.float32(2.0 ** -8))]], np.uint16)
    b1 = np.array([[O.f32_to_bf16(np.float32(1.0))]], np.uint16)
    assert O.dequant4_bf16(w1, s1, b1)[0, 0] == O.f32_to_bf16(np.float32(1.0))


def test_golden_rmsnorm_order(golden):
    """The MoE stack's layer-input RMSNorm follows rmsnorm.metal's reduction order
    exactly: with the oracle's fp32 rms, x / rms rounded to f16 reproduces the
    reference kernel's f16 output bit for bit."""
    g = golden("rmsnorm")
    x = g["x"]
    rms = O.rms_layer(x)
    v = O.bf16_to_f32(x) / rms[:, None]
    assert v.dtype == np.float32
    assert np.array_equal(v.astype(np.float16).view(np.uint16), g["out"].view(np.uint16))
    assert np.array_equal(O.rmsnorm_layer(x), O.f32_to_bf16(v))


def test_routing_agreement_with_reference_on_config1():
    """Config 1's 512 tokens routed by the oracle (fp32 logits, selection on logits) and by
    the reference's own kernels (logits rounded to f16, dequant_matvec_8bit.metal:30;
    selection on probabilities with the lowest index winning ties,
    moe_routing_topk.metal:43-52).  Pinned: 4 of the 512 tokens get a different top-8
    set, each by one expert, and at every such token the two experts' f16 logits are
    equal -- a tie the reference's rounding creates and its lowest-index rule breaks,
    where the unrounded fp32 logits still tell the experts apart."""
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built")
    L = O.synth_layer(0, 0)
    x = O.synth_x(0, 0, 512, 2048)
    rl, rid, _ = O.ref_route(L, x)
    lg = O.router_logits(L, x)
    oid, _ = O.topk(lg, 8)
    differ = [t for t in range(512) if set(oid[t]) != set(rid[t])]
    assert len(differ) == 4, differ
    for t in differ:
        only_o, only_r = set(oid[t]) - set(rid[t]), set(rid[t]) - set(oid[t])
        assert len(only_o) == len(only_r) == 1
        a, b = only_o.pop(), only_r.pop()
        assert rl[t, a] == rl[t, b]            # tied after the reference's f16 rounding
        assert b < a                           # ... and broken by the lower index
        assert lg[t, a] > lg[t, b]             # the fp32 logits order them the other way
    # where the sets agree, the ranks agree too except within such f16 ties
    same = [t for t in range(512) if t not in differ]
    for t in same:
        if not np.array_equal(oid[t], rid[t]):
            for k in range(8):
                if oid[t, k] != rid[t, k]:
                    assert rl[t, oid[t, k]] == rl[t, rid[t, k]]


def test_embed_is_the_reference_row_dequant():
    """Model::embed (src/forward.rs:449-460): w = nib * scale + bias in f32 per column,
    nibble (word >> 4*(i % 8)) & 15; the oracle rounds that f32 value to bf16 once."""
    hd = O.synth_head(2, vocab=512)
    toks = np.array([0, 7, 511, 300], np.int32)
    got = O.embed(hd, toks)
    for r, tok in enumerate(toks):
        words = hd.embed_w[tok]
        nib = np.array([(words[i // 8] >> (4 * (i % 8))) & 0xF for i in range(2048)], np.float32)
        sc = np.repeat(O.bf16_to_f32(hd.embed_s[tok]), 64)
        bi = np.repeat(O.bf16_to_f32(hd.embed_b[tok]), 64)
        ref = (nib * sc + bi).astype(np.float32)   # q*s is exact in fp32: one rounding, as fmaf
        assert np.array_equal(got[r], O.f32_to_bf16(ref))


def test_lm_head_argmax_agrees_with_the_reference_kernels():
    """The end of run_one_token (src/forward.rs:553-566) by the reference's own kernels
    (rmsnorm.metal, fused_dequant_matvec_4bit.metal in f16, then the CPU scan where the
    first maximum wins) against the oracle's canonical fp32 order: on 32 tokens over a
    vocabulary of 8,192 rows the next token agrees for every token (pinned), and the
    logits agree within 4e-3 of the largest."""
    R = O.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built")
    hd = O.synth_head(0, vocab=8192)
    T = 32
    x = O.synth_x(0, 0, T, 2048)
    lg, ids = O.lm_head(hd, x, nthreads=4)
    f16 = lambda a: O.bf16_to_f32(a).astype(np.float16)  # noqa: E731
    xn = np.empty((T, 2048), np.float16)
    R.ref_rmsnorm(np.ascontiguousarray(f16(x)), np.ascontiguousarray(f16(hd.norm_w)), xn, T, 2048, 1e-6)
    rl = np.empty((T, 8192), np.float16)
    for t in range(T):
        R.ref_fused_dequant_matvec_4bit(hd.lm_w, f16(hd.lm_s), f16(hd.lm_b), np.ascontiguousarray(xn[t]), rl[t],
                                        2048, 8192, 4)
    rid = np.array([int(np.argmax(r.astype(np.float32))) for r in rl], np.int32)
    assert np.array_equal(rid, ids)
    assert np.abs(rl.astype(np.float32) - lg).max() <= 4e-3 * np.abs(lg).max()
