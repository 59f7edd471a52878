"""The attention oracle (oracle/obs_oracle.c orc_attn_forward) pinned against
the reference's own kernels run on the CPU: rmsnorm.metal, fused 4-bit mat-vecs,
rope.metal, ops.metal kv_append / ew_add and sdpa_decode.metal strung together
as Model::forward_layer does (src/forward.rs:404-419), one decode token at a
time.  The oracle works in bf16 and the reference in f16, so the pins are
normwise (max |d| / max |ref|) within the 1e-2 contract; the oracle's own
batching rules (prefill == token by token, interleaved sequences == separate
ones) are bit-exact."""
import numpy as np
import pytest

import oracle as O
from parity_util import REL, rel_err as normwise

TOL = REL  # the north star's bf16 contract
pytestmark = pytest.mark.skipif(O.ref_lib() is None, reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def attn():
    return O.synth_attn(seed=5, layer=0)


def _f(a):
    return a.astype(np.float32) if a.dtype in (np.float16, np.float32) else O.bf16_to_f32(a)


def test_prefill_matches_reference_token_by_token(attn):
    P = 24
    x = O.synth_x(5, 0, P, attn.H)
    st = O.AttnState(attn, 64, 1)
    out = st.forward(x, np.zeros(P, np.int32), np.arange(P, dtype=np.int32))
    ref = O.RefAttnState(attn, 64)
    r = np.stack([ref.token(x[i], i) for i in range(P)])
    assert normwise(_f(out), _f(r)) < TOL
    # the attention's contribution alone (out - x), same bound
    assert normwise(_f(out) - _f(x), _f(r) - _f(x)) < TOL
    # the caches the block appended: k after head norm and RoPE, v raw
    assert normwise(_f(st.kc[0][:, :P]), _f(ref.kc[:, :P])) < TOL
    assert normwise(_f(st.vc[0][:, :P]), _f(ref.vc[:, :P])) < TOL


@pytest.mark.parametrize("positions", [[0, 1, 4999, 40959], [17, 30000]])
def test_long_positions_match_reference(attn, positions):
    """Tokens written at far positions of a zeroed cache (both sides attend to the
    zero rows in between the same way): the table RoPE (double-precision angles)
    against rope.metal's fp32 pow/cos/sin at positions up to the model's maximum."""
    n = len(positions)
    x = O.synth_x(6, 0, n, attn.H)
    st = O.AttnState(attn, 40960, 1)
    ref = O.RefAttnState(attn, 40960)
    for i, p in enumerate(positions):
        o = st.forward(x[i:i + 1], np.zeros(1, np.int32), np.array([p], np.int32))
        r = ref.token(x[i], p)
        assert normwise(_f(o[0]), _f(r)) < TOL, p
        assert normwise(_f(st.kc[0][:, p]), _f(ref.kc[:, p])) < TOL, p


def test_rope_matches_reference_shader():
    """The oracle's rotation (cos/sin table, a = x1 s, fmaf(x0, c, -a), ...) against
    rope.metal on the same head rows, inputs exact in both bf16 and f16."""
    rng = np.random.default_rng(3)
    hd, nh = 128, 8
    xb = O.f32_to_bf16(rng.standard_normal((nh, hd)).astype(np.float32))
    for pos in (0, 1, 7, 1000, 40959):
        tab = np.empty((pos + 1, hd // 2, 2), np.float32)
        O.lib().orc_rope_table(1e7, hd, pos + 1, tab)
        c, s = tab[pos, :, 0], tab[pos, :, 1]
        x = O.bf16_to_f32(xb)
        x0, x1 = x[:, :hd // 2], x[:, hd // 2:]
        mine = np.concatenate([x0 * c - x1 * s, x1 * c + x0 * s], axis=1)
        r = O.ref_rope(O.bf16_to_f32(xb).astype(np.float16), pos).astype(np.float32)
        assert normwise(mine, r) < 2e-3, pos


def test_rope_table_is_the_double_precision_angle():
    hd, n = 128, 300
    tab = np.empty((n, hd // 2, 2), np.float32)
    O.lib().orc_rope_table(1e7, hd, n, tab)
    ang = np.arange(n)[:, None] * np.power(1e7, -2.0 * np.arange(hd // 2) / hd)[None, :]
    assert np.array_equal(tab[..., 0], np.cos(ang).astype(np.float32))
    assert np.array_equal(tab[..., 1], np.sin(ang).astype(np.float32))


def test_oracle_batching_is_exact(attn):
    """A chunked prefill equals the one-call prefill, and one call carrying tokens of
    two sequences equals the two sequences run separately (bit-exact)."""
    xa = O.synth_x(7, 0, 10, attn.H)
    xb = O.synth_x(8, 0, 6, attn.H)
    one = O.AttnState(attn, 32, 2)
    oa = one.forward(xa, np.zeros(10, np.int32), np.arange(10, dtype=np.int32))
    ob = one.forward(xb, np.ones(6, np.int32), np.arange(6, dtype=np.int32))
    two = O.AttnState(attn, 32, 2)
    c1 = two.forward(xa[:4], np.zeros(4, np.int32), np.arange(4, dtype=np.int32))
    mix_x = np.concatenate([xa[4:], xb])
    mix_s = np.array([0] * 6 + [1] * 6, np.int32)
    mix_p = np.concatenate([np.arange(4, 10), np.arange(6)]).astype(np.int32)
    c2 = two.forward(mix_x, mix_s, mix_p)
    assert np.array_equal(np.concatenate([c1, c2[:6]]), oa)
    assert np.array_equal(c2[6:], ob)
    assert np.array_equal(one.kc, two.kc) and np.array_equal(one.vc, two.vc)
