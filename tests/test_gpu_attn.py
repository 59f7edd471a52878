"""The attention block on the GPU (obs_attn_forward) against the oracle at the
Qwen3-30B-A3B shape: H 2048, 32 query heads, 4 KV heads, head_dim 128,
rope_theta 1e7.  A session of three sequences: a prefill, a chunked prefill,
batched decode steps mixing the sequences, and a token at the cache's last
position.  The K and V caches are bit-exact (projections in the canonical fp32
order, head norm, table RoPE); the outputs differ from the oracle only in the
softmax's exponential, its sum order and one division, so they are compared
normwise within 5e-3 (the whole output) and 1e-2 (the attention's contribution,
out - x)."""
import numpy as np
import pytest

import obsmoe
import oracle as O
from parity_util import REL, REL_SAME, dev, host, rel_err

pytestmark = pytest.mark.gpu

H, NQ, NKV, HD, THETA = 2048, 32, 4, 128, 1e7
MAX_SEQ, N_SEQS = 512, 3


@pytest.fixture(scope="module")
def attn(cuda):
    A = O.synth_attn(seed=9, layer=0, H=H, nq=NQ, nkv=NKV, hd=HD)
    ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, 768, 128, 8, n_layers=1, max_tokens=64), 0)
    ctx.attn_init(NQ, NKV, HD, MAX_SEQ, N_SEQS, THETA)
    ctx.load_attn(0, A)
    yield cuda, ctx, A
    ctx.close()


def _step(torch, ctx, st, x, seq, pos):
    T = len(seq)
    out = torch.empty((T, H), dtype=torch.int16, device="cuda")
    ctx.attn_forward(0, dev(torch, x), out, T, dev(torch, np.array(seq, np.int32)),
                     dev(torch, np.array(pos, np.int32)))
    ctx.check_device()
    got = host(out, np.uint16)
    ref = st.forward(x, np.array(seq, np.int32), np.array(pos, np.int32))
    xf = O.bf16_to_f32(x)
    return rel_err(got, ref), rel_err(O.bf16_to_f32(got) - xf, O.bf16_to_f32(ref) - xf)


def test_attention_session_matches_oracle(attn):
    torch, ctx, A = attn
    st = O.AttnState(A, MAX_SEQ, N_SEQS, THETA)
    lens = [0, 0, 0]
    steps = []
    # a 40-token prefill of sequence 0; a prefill of sequence 1 in two chunks
    steps.append(([0] * 40, list(range(40))))
    steps.append(([1] * 10, list(range(10))))
    steps.append(([1] * 7, list(range(10, 17))))
    # five batched decode steps over all three sequences
    for i in range(5):
        steps.append(([0, 1, 2], [40 + i, 17 + i, i]))
    # sequence 2 jumps to the cache's last position (the rows in between stay zero on both sides)
    steps.append(([2], [MAX_SEQ - 1]))
    for k, (seq, pos) in enumerate(steps):
        x = O.synth_x(100 + k, 0, len(seq), H)
        whole, delta = _step(torch, ctx, st, x, seq, pos)
        assert whole <= REL_SAME, (k, whole)
        assert delta <= REL, (k, delta)
        for s, p in zip(seq, pos):
            lens[s] = max(lens[s], p + 1)
    # every cache row written, bit for bit
    for s in range(N_SEQS):
        kc = torch.empty((NKV, MAX_SEQ, HD), dtype=torch.int16, device="cuda")
        vc = torch.empty_like(kc)
        ctx.kv_read(0, s, 0, MAX_SEQ, kc, vc)
        torch.cuda.synchronize()
        assert np.array_equal(host(kc, np.uint16), st.kc[s]), s
        assert np.array_equal(host(vc, np.uint16), st.vc[s]), s


def test_attention_refuses_out_of_range_positions(attn):
    """A position at max_seq (or a sequence id past n_seqs) is refused by the kernel's
    bounds check: nothing is written and the context reports it."""
    torch, ctx, A = attn
    x = dev(torch, O.synth_x(200, 0, 1, H))
    out = torch.empty((1, H), dtype=torch.int16, device="cuda")
    for seq, pos in ((0, MAX_SEQ), (N_SEQS, 0), (0, -1)):
        ctx.attn_forward(0, x, out, 1, dev(torch, np.array([seq], np.int32)), dev(torch, np.array([pos], np.int32)))
        with pytest.raises(obsmoe.ObsError, match="outside the KV caches"):
            ctx.check_device()
    ctx.check_device()  # the flag was cleared


def test_attention_host_errors(attn):
    torch, ctx, A = attn
    x = torch.zeros((65, H), dtype=torch.int16, device="cuda")
    s = torch.zeros(65, dtype=torch.int32, device="cuda")
    with pytest.raises(obsmoe.ObsError, match="T out of range"):
        ctx.attn_forward(0, x, x, 65, s, s)
    with pytest.raises(obsmoe.ObsError, match="alias"):
        ctx.attn_forward(0, x, x, 1, s, s)
    with pytest.raises(obsmoe.ObsError, match="layer out of range"):
        ctx.attn_forward(1, x, x, 1, s, s)
    with pytest.raises(obsmoe.ObsError, match="already initialised"):
        ctx.attn_init(NQ, NKV, HD, MAX_SEQ, N_SEQS, THETA)
    c2 = obsmoe.MoeContext(obsmoe.MoeShape(H, 768, 128, 8, n_layers=1, max_tokens=4), 0)
    with pytest.raises(obsmoe.ObsError, match="not initialised"):
        c2.attn_forward(0, x, x, 1, s, s)
    with pytest.raises(obsmoe.ObsError, match="bad attention config"):
        c2.attn_init(NQ, 5, HD, MAX_SEQ, 1, THETA)
    with pytest.raises(obsmoe.ObsError, match="bad attention config"):
        c2.attn_init(NQ, 2, HD, MAX_SEQ, 1, THETA)  # 16 query heads per KV head: more than one CTA takes
    with pytest.raises(obsmoe.ObsError, match="bad attention config"):
        c2.attn_init(NQ, NKV, HD, 40961, 1, THETA)
    c2.close()
