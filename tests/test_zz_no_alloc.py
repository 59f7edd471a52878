"""obs_decode_ffn_static: the decode expert FFN for callers that cannot
allocate device memory (code running while a CUDA graph is being captured,
frameworks that own every device byte through their own arena, loops that
cannot afford an allocation's implicit synchronisation).  Its scratch is a
fixed array inside the library, so it needs no context.

Checked through the C ABI, on two calls in a row (they share the library's
array, which keeps the previous call's contents):
* bit for bit against the context's decode path on the same routes (the two
  run the same arithmetic in the same order), where the context takes the shape;
* against the CPU oracle, on every shape, including the limits the header
  states (T * top_k = 64, hidden 4096, inter 1536) and the smallest hidden and
  inter (512 and 128), with the output pre-filled with a sentinel so an element
  the kernels never write cannot pass.
This file runs last in the suite and also passes on its own in a fresh process."""
import numpy as np
import pytest

import obsmoe
import oracle as O
from parity_util import REL, REL_ELEM, dev, elem_err, rel_err

pytestmark = pytest.mark.gpu

SENTINEL = 0x7FC1  # a bf16 NaN: never a result of the kernels


class DevWeights:
    """Expert weights of one layer on the device, in the reference (MLX) layout."""

    def __init__(self, torch, L):
        for n in ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s", "down_b"):
            setattr(self, n, dev(torch, getattr(L, n)))


def routes(rng, T, E, K):
    ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32) + 0.05
    return ids, (w / w.sum(1, keepdims=True)).astype(np.float32)


# (E, H, I, K, T, context): context = the context path accepts the shape (hidden a
# multiple of 2048, inter a multiple of 256), so the bit-exact comparison runs too
CASES = [
    (16, 2048, 256, 4, 6, True),
    (32, 2048, 768, 8, 8, True),      # Qwen3-30B-A3B's expert shape at T * top_k = 64
    (8, 4096, 1536, 8, 8, True),      # hidden and inter at their maxima, T * top_k = 64
    (8, 512, 256, 1, 64, False),      # the smallest hidden, T * top_k = 64
    (8, 2048, 128, 8, 1, False),      # the smallest inter: 64-thread down blocks
]


@pytest.mark.parametrize("E,H,I,K,T,with_ctx", CASES)
def test_decode_ffn_static(cuda, E, H, I, K, T, with_ctx):
    torch = cuda
    L = O.synth_layer(31, 0, E=E, H=H, I=I, K=K)
    w = DevWeights(torch, L)
    ctx = None
    if with_ctx:
        ctx = obsmoe.MoeContext(obsmoe.MoeShape(H, I, E, K, n_layers=1, max_tokens=max(T, 16)), 0)
        ctx.load_layer(0, L)
    rng = np.random.default_rng(E * 1000 + T)
    for call in range(2):  # two calls in a row share the library's scratch
        xh = O.synth_x(31, 0, T, H, row0=100 * call)
        resh = O.synth_x(32, 0, T, H, row0=100 * call) if call == 1 else None
        ids_h, wts_h = routes(rng, T, E, K)
        x, ids, wts = dev(torch, xh), dev(torch, ids_h), dev(torch, wts_h)
        res = None if resh is None else dev(torch, resh)
        out = torch.full((T, H), SENTINEL, dtype=torch.int16, device="cuda")
        obsmoe.decode_ffn_static(w, E, H, I, K, x, ids, wts, T, out, residual=res)
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        assert not np.any(got == SENTINEL), f"call {call}: elements left unwritten"
        ref, _, _ = O.moe_ffn_combine(L, xh, ids_h, wts_h, residual=resh, wmode=0)
        assert rel_err(got, ref) < REL, f"call {call}"
        assert elem_err(got, ref) < REL_ELEM, f"call {call}"
        if ctx is not None:
            # the existing entry point on the same routes: the context's decode FFN
            y = torch.empty((T * K, H), dtype=torch.int16, device="cuda")
            ctx.expert_ffn(0, x, ids, T, y, path=obsmoe.PATH_DECODE)
            torch.cuda.synchronize()
            yh = O.bf16_to_f32(y.cpu().numpy().view(np.uint16)).reshape(T, K, H)
            # the combine in rank order, fp32, one rounding (the kernels' own order)
            acc = np.zeros((T, H), np.float32) if resh is None else O.bf16_to_f32(resh).copy()
            for k in range(K):
                acc = (wts_h[:, k:k + 1].astype(np.float32) * yh[:, k] + acc).astype(np.float32)
            mine = O.bf16_to_f32(got)
            assert rel_err(mine, acc) < 2 ** -7, f"call {call}"
            full = torch.empty((T, H), dtype=torch.int16, device="cuda")
            y_static = torch.empty((T * K, H), dtype=torch.int16, device="cuda")
            # bit for bit: the context's decode FFN rows against the static entry's, one rank at a time
            for k in range(K):
                onehot = np.zeros((T, K), np.float32)
                onehot[:, k] = 1.0
                obsmoe.decode_ffn_static(w, E, H, I, K, x, ids, dev(torch, onehot), T, full)
                y_static.view(T, K, H)[:, k].copy_(full)
            torch.cuda.synchronize()
            assert torch.equal(y_static, y), f"call {call}: static and context decode FFN differ"
    if ctx is not None:
        ctx.check_device()
        ctx.close()


def test_decode_ffn_static_rejects_oversize(cuda):
    torch = cuda
    E, H, I, K = 16, 2048, 256, 4
    L = O.synth_layer(31, 0, E=E, H=H, I=I, K=K)
    w = DevWeights(torch, L)
    T = 17  # T * K = 68 > OBS_STATIC_MAX_PAIRS
    x = torch.zeros((T, H), dtype=torch.int16, device="cuda")
    ids = torch.zeros((T, K), dtype=torch.int32, device="cuda")
    wts = torch.zeros((T, K), dtype=torch.float32, device="cuda")
    with pytest.raises(obsmoe.ObsError, match="OBS_STATIC_MAX_PAIRS"):
        obsmoe.decode_ffn_static(w, E, H, I, K, x, ids, wts, T, x)
    with pytest.raises(obsmoe.ObsError, match="inter"):
        obsmoe.decode_ffn_static(w, E, H, 4096, K, x[:2], ids[:2], wts[:2], 2, x[:2])
    with pytest.raises(obsmoe.ObsError, match="hidden"):
        obsmoe.decode_ffn_static(w, E, 8192, I, K, x[:1], ids[:1], wts[:1], 1, x[:1])
